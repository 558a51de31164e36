/*
 * ggmlc_b200 — C ABI of the B200 execution engine for ggmlc-compiled GGUF decoder graphs.
 *
 * This is the drop-in boundary that replaces the reference's nanobind module `ggmlc._runtime`
 * (runtime/bindings/python_bindings.cpp:22-295) for the CUDA hot path.  Each entry point names
 * the binding it replaces.  Plain C types only: opaque handles, pointers and sizes.
 *
 * Conventions: functions return 0 on success and -1 on error; gb_last_error() then holds the
 * message (thread-local).  Strings returned by the library stay valid until the owning handle
 * is freed or the same call is made again.  Host buffers passed in are only read during the
 * call.  Device pointers (the op-level section) must be CUDA device memory of the current
 * device; `stream` is a cudaStream_t (NULL = legacy default stream).
 */
#ifndef GGMLC_B200_H
#define GGMLC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gb_graph gb_graph;       /* ggmlc::SerializedModelGraph */
typedef struct gb_executor gb_executor; /* ggmlc::ModelExecutor */

/* Last error message of this thread ("" if none). */
const char* gb_last_error(void);
/* ABI version (major * 10000 + minor * 100 + patch). */
int gb_version(void);

/* get_available_devices() — python_bindings.cpp:133: "cpu", "cuda:0".., "cuda".  Writes a
 * '\n'-separated list into buf (capacity cap); returns the needed length or -1. */
int gb_get_available_devices(char* buf, size_t cap);

/* ---- ModelLoader (python_bindings.cpp:108-130; loader.cpp:257-443) ------------------------ */
int gb_loader_load_from_file(const char* path, gb_graph** out);
int gb_loader_load_from_bytes(const void* data, size_t size, gb_graph** out);
void gb_graph_free(gb_graph* g);

/* SerializedModelGraph fields (python_bindings.cpp:71-106) */
const char* gb_graph_name(const gb_graph* g);
int gb_graph_num_symbols(const gb_graph* g);
const char* gb_graph_symbol(const gb_graph* g, int i);
/* which: 0 inputs, 1 outputs, 2 parameters */
int gb_graph_num_ids(const gb_graph* g, int which);
int gb_graph_id(const gb_graph* g, int which, int i, uint32_t* id);
int gb_graph_num_tensors(const gb_graph* g);
int gb_graph_tensor_id(const gb_graph* g, int i, uint32_t* id);
/* SerializedTensor(id, name, data_size, storage, type) — python_bindings.cpp:71-92 */
int gb_graph_tensor_info(const gb_graph* g, uint32_t id, const char** name, int* type,
                         int* storage, uint64_t* data_size);
/* SerializedTensor.symbol_index(axis): symbol-table index of dim `axis`, or -1 */
int gb_graph_tensor_symbol_index(const gb_graph* g, uint32_t id, int axis);
int gb_graph_num_ops(const gb_graph* g);
int gb_graph_op_info(const gb_graph* g, int i, uint32_t* id, int* opcode, const char** name);
/* metadata string (e.g. "general.name"); NULL when absent */
const char* gb_graph_metadata_str(const gb_graph* g, const char* key);

/* ---- ModelExecutor (python_bindings.cpp:136-217; executor.h:25-287) ----------------------- */
/* device: "cuda", "cuda:N" or "auto".  "cpu" is refused: this engine has no CPU fallback. */
int gb_executor_create(const gb_graph* g, const char* device, gb_executor** out);
/* Tensor parallelism (no counterpart in the reference, which runs one device per model).
 * gb_nccl_unique_id writes the 128-byte NCCL unique id that rank 0 creates and the caller
 * shares with every rank; gb_executor_create_tp then builds rank tp_rank of a tp_size-way
 * group on `device` (collective: all ranks must call it).  Fused QKV is cut by heads, fused
 * gate_up per half, O / down along K with an all-reduce of their partial sums, the output
 * projection by vocabulary rows with an all-gather of the logits; each rank uploads only its
 * weight slices and keeps its own KV heads.  Outputs are complete on every rank.
 * gb_tp_plan returns, without touching a device, the plan of one rank as JSON (weight slices,
 * partial-sum tensors, rewritten shapes) or NULL (gb_last_error) for unsupported graphs. */
int gb_nccl_unique_id(void* out128);
int gb_executor_create_tp(const gb_graph* g, const char* device, int tp_rank, int tp_size,
                          const void* nccl_id, gb_executor** out);
const char* gb_tp_plan(const gb_graph* g, int tp_rank, int tp_size);
int gb_executor_tp_size(const gb_executor* e);
/* Decode-sized partial sums are summed by a one-shot all-reduce over peer memory (CUDA IPC,
 * NVLink stores, bounded waits); gb_executor_tp_error returns 0 while every such wait
 * completed, 1 once one gave up on a peer (that call's sum is not valid), -1 on error.  The
 * executor also checks the word at every host synchronisation (gb_executor_synchronize and
 * every output read): a wait that gave up makes that call fail with an error naming it
 * (gb_last_error), once, and clears the word. */
int gb_executor_tp_error(gb_executor* e);
int gb_executor_tp_rank(const gb_executor* e);
void gb_executor_free(gb_executor* e);
const char* gb_executor_device(const gb_executor* e);
/* prepare(symbols, enable_arena_reuse) — executor.cpp:1453 */
int gb_executor_prepare(gb_executor* e, const char* const* names, const int64_t* values, int n,
                        int enable_arena_reuse);
/* set_input_by_id / set_input_by_name — executor.cpp:2928-2944 (host -> device copy) */
int gb_executor_set_input(gb_executor* e, uint32_t tid, const void* data, size_t bytes);
int gb_executor_set_input_by_name(gb_executor* e, const char* name, const void* data,
                                  size_t bytes);
/* run(n_threads) — executor.cpp:2984 (n_threads is accepted and ignored on the GPU) */
int gb_executor_run(gb_executor* e, int n_threads);
int gb_executor_synchronize(gb_executor* e);
/* get_output_bytes — executor.cpp:3138-3157: device -> host copy; *data is owned by the
 * executor and valid until the next call for the same tensor */
int gb_executor_get_output(gb_executor* e, uint32_t tid, const void** data, size_t* bytes);
/* Engine extension, no reference twin: the greedy token (first maximum) of each of `rows` rows
 * of an f32 output [rows][n], computed on the device; only the `rows` indices cross to the host
 * (the reference's runner copies the logits and takes the argmax on the host). */
int gb_executor_output_argmax(gb_executor* e, uint32_t tid, int rows, int32_t* out);
int gb_executor_get_tensor_shape(gb_executor* e, uint32_t tid, int64_t ne[4]);
int gb_executor_get_tensor_size_bytes(gb_executor* e, uint32_t tid, size_t* bytes);
/* set_state_by_id / get_state_bytes / reset_state — executor.cpp:3063-3136 */
int gb_executor_set_state(gb_executor* e, uint32_t tid, const void* data, size_t bytes);
int gb_executor_get_state(gb_executor* e, uint32_t tid, const void** data, size_t* bytes);
int gb_executor_reset_state(gb_executor* e);
/* init_kv_cache / reset_kv_cache / has_kv_cache — executor.cpp:498-632 */
int gb_executor_init_kv_cache(gb_executor* e, int64_t max_ctx);
int gb_executor_reset_kv_cache(gb_executor* e);
int gb_executor_has_kv_cache(const gb_executor* e);
/* set_logits_last_only / logits_last_only — executor.cpp:2398-2410 */
int gb_executor_set_logits_last_only(gb_executor* e, int enable);
/* Output rows (the per-request output indices of the reference's doc gap 3, "Multi-request
 * outputs", docs/benchmarks/ggmlc_vs_llama_cpp.md:195; llama's out_ids): the next prefills
 * compute their output projections for rows[0..n) of the call's tokens only, in that order
 * (n <= 64, each below the call's token count, checked at prepare); logits come back as
 * [n][vocab].  n = 0 turns it off.  Takes precedence over set_logits_last_only. */
int gb_executor_set_output_rows(gb_executor* e, const int32_t* rows, int n);
int gb_executor_logits_last_only(const gb_executor* e);
/* set_enable_cuda_graph / is_cuda_graph_enabled / is_cuda_graph_captured — cuda_graph.cu */
int gb_executor_set_enable_cuda_graph(gb_executor* e, int enable);
int gb_executor_is_cuda_graph_enabled(const gb_executor* e);
int gb_executor_is_cuda_graph_captured(const gb_executor* e);
/* Decode chains (engine switch, no reference twin): a single-sequence decode step on one GPU
 * runs its GEMVs, attention and row norms as ONE persistent launch (one CTA per SM, grid
 * barriers between ops, weight copies requested ahead across op boundaries).  Off by default
 * (environment GGMLC_B200_CHAIN=1 turns the default on where the device supports cooperative
 * launch); changing it drops the prepared programs.  A chain wait that runs out (about 2 s)
 * makes the next output read raise, and later chain launches in the process do nothing. */
int gb_executor_set_decode_chain(gb_executor* e, int enable);
int gb_executor_decode_chain(const gb_executor* e);
/* set_enable_profile / reset_profile / get_profile — executor.h:103-116 */
int gb_executor_set_enable_profile(gb_executor* e, int enable);
int gb_executor_reset_profile(gb_executor* e);
int gb_executor_get_profile(gb_executor* e, double* prepare_ms, double* run_ms, int* n_prepare,
                            int* n_run);
/* runtime_graph_summary / runtime_mul_mat_shape_summary — executor.cpp:3211-3459 (JSON) */
const char* gb_executor_graph_summary(gb_executor* e);
const char* gb_executor_mul_mat_shape_summary(gb_executor* e);
/* kernel launches per run() of the prepared program (engine telemetry, no reference twin) */
int64_t gb_executor_launches_per_run(const gb_executor* e);
/* per-launch device timing for roofline accounting (engine telemetry; the reference's nearest
 * twin is ExecutorProfile, executor.h:103-116): while enabled, run() brackets each launch with
 * CUDA events; gb_executor_kernel_times returns JSON {name: [ms, launches, algorithmic bytes]} */
int gb_executor_set_kernel_timing(gb_executor* e, int enable);
int gb_executor_reset_kernel_times(gb_executor* e);
const char* gb_executor_kernel_times(gb_executor* e);
/* the executor's CUDA stream (cudaStream_t), for callers that order their own work after it */
void* gb_executor_stream(const gb_executor* e);

/* ---- paged KV cache (python_bindings.cpp:196-204; executor.cpp:634-920) ---------------------
 * init_paged_kv_cache(max_batch, max_ctx): max_batch sequence slots (1..16) of up to max_ctx
 * positions over a pool of pages.  A page holds tokens_per_page positions (a power of two) of K
 * and V in every attention layer; each layer's pool is [page][Hkv][tokens_per_page][head_dim]
 * fp16 and a device page table maps each slot's runs of positions to pages (the reference maps
 * driver-VMM pages into per-slot address windows instead; here the kernels read the table).
 * paged_kv_ensure_tokens assigns pages as a slot grows, paged_kv_free_slot returns them, and
 * paged_active_vram_bytes counts the pages mapped into slots.  prepare() with symbol "slot"
 * runs a single sequence in that slot (its positions must have pages); gb_executor_prepare_batch
 * runs one decode token for each of `rows` sequences (row r at position pos[r] in slot
 * slot[r]; slot == max_batch is a scratch slot for padding rows).  set_tokens_per_page on an
 * initialised cache lays the pool out again and needs every slot free. */
int gb_executor_init_paged_kv_cache(gb_executor* e, int64_t max_batch, int64_t max_ctx);
int gb_executor_is_paged_kv_cache_enabled(const gb_executor* e);
int gb_executor_paged_kv_alloc_slot(gb_executor* e, int64_t slot);
int gb_executor_paged_kv_free_slot(gb_executor* e, int64_t slot);
int gb_executor_paged_kv_ensure_tokens(gb_executor* e, int64_t slot, int64_t total_tokens);
int64_t gb_executor_paged_active_vram_bytes(const gb_executor* e);
int64_t gb_executor_tokens_per_page(const gb_executor* e);
int gb_executor_set_tokens_per_page(gb_executor* e, int64_t tokens_per_page);
int gb_executor_prepare_batch(gb_executor* e, int rows, const int32_t* pos, const int32_t* slot);

/* Pool size, read at the next init_paged_kv_cache.  configure_prefix_pool (configure_vmm_pool's
 * max_warm_pages, python_bindings.cpp:201): pages kept for the prefix cache on top of max_batch
 * full sequences; 0 (default): about 2 GiB of pages, at most max_batch sequences' worth.  Cached
 * prefix pages are shared with the slots that use them (a reference each, no copy).
 * configure_kv_pool_pages: the pool's exact page count instead (0: the rule above); a pool
 * smaller than max_batch full sequences makes the scheduler admit requests as pages allow.
 * kv_pool_pages / kv_free_pages: pages of the current pool / pages nobody references. */
int gb_executor_configure_prefix_pool(gb_executor* e, int64_t pages);
int gb_executor_configure_kv_pool_pages(gb_executor* e, int64_t pages);
int64_t gb_executor_kv_pool_pages(const gb_executor* e);
int64_t gb_executor_kv_free_pages(const gb_executor* e);

/* ---- PagedRadixTree (radix_tree.h; radix_tree.cpp:7-220; python_bindings.cpp:248-258) -------
 * Prefix index over whole pages of tokens_per_page tokens: 64-bit FNV-1a chunk hashes verified
 * token by token, least-recently-used leaf eviction.  Standalone handle for tests and callers;
 * the scheduler keeps its own.  insert_prefix attaches the whole pages of `tokens` not yet
 * present (page ids 0, 1, 2, ... in insertion order); evict_lru returns the freed page id or
 * -1. */
typedef struct gb_radix gb_radix;
int gb_radix_create(int64_t tokens_per_page, gb_radix** out);
void gb_radix_free(gb_radix* r);
int64_t gb_radix_tokens_per_page(const gb_radix* r);
int64_t gb_radix_total_cached_pages(const gb_radix* r);
int64_t gb_radix_total_nodes(const gb_radix* r);
void gb_radix_reset(gb_radix* r);
int gb_radix_match_prefix(gb_radix* r, const int32_t* tokens, int64_t n, int64_t* matched_pages,
                          int64_t* matched_tokens);
int gb_radix_insert_prefix(gb_radix* r, const int32_t* tokens, int64_t n, int64_t* added);
int64_t gb_radix_evict_lru(gb_radix* r);

/* ---- ContinuousBatchScheduler (batch_scheduler.h:35-77; python_bindings.cpp:261-295) --------
 * Iteration-level continuous batching over the paged KV cache: add_request queues a prompt
 * (refused if prompt + max_new_tokens exceed max_ctx or the pool's pages); each step either
 * admits, in order, every pending request that finds a free slot and whose pages fit the pool
 * next to what the running sequences may still claim (prefill into it, first token;
 * batch_scheduler.cpp:136-277), or decodes one token for every active sequence at its own
 * position.  Greedy when temperature <= 0.  Prefix caching (on by default): the pages of the
 * longest cached run of whole prompt pages are mapped into the slot's page table (shared, not
 * copied) and only the rest of the prompt is prefilled (batch_scheduler.cpp:149-164,
 * :225-238); least-recently-used cached pages are evicted when admission needs their room. */
typedef struct gb_scheduler gb_scheduler;
typedef struct gb_request_info {
    uint64_t request_id;
    int slot_id;
    int64_t current_pos;
    int max_new_tokens;
    float temperature;
    int eos_token_id;
    int finished;
    const char* finish_reason; /* "stop", "length" or "" (valid while the scheduler lives) */
    int64_t n_prompt_tokens;
    int64_t n_generated_tokens;
    int64_t prefix_tokens_matched;
} gb_request_info;
int gb_scheduler_create(gb_executor* e, int max_batch_size, int eos_token_id, gb_scheduler** out);
void gb_scheduler_free(gb_scheduler* s);
int gb_scheduler_add_request(gb_scheduler* s, const int32_t* prompt, int64_t n, int max_new_tokens,
                             float temperature, int eos_token_id, uint64_t* request_id);
/* new tokens as (ids[i], tokens[i]), i < *n_new; completed request ids in done[j], j < *n_done */
int gb_scheduler_step(gb_scheduler* s, uint64_t* ids, int32_t* tokens, int cap, int* n_new,
                      uint64_t* done, int cap_done, int* n_done);
int gb_scheduler_has_work(const gb_scheduler* s);
int64_t gb_scheduler_active_count(const gb_scheduler* s);
int64_t gb_scheduler_pending_count(const gb_scheduler* s);
int gb_scheduler_max_batch_size(const gb_scheduler* s);
int gb_scheduler_enable_prefix_caching(gb_scheduler* s, int enable);
int gb_scheduler_is_prefix_caching_enabled(const gb_scheduler* s);
/* total_prefix_cache_hits / total_prefix_tokens_saved (batch_scheduler.h:56-57) */
int gb_scheduler_prefix_stats(const gb_scheduler* s, int64_t* hits, int64_t* tokens_saved);
int gb_scheduler_get_request(gb_scheduler* s, uint64_t request_id, gb_request_info* info);
/* which: 0 prompt tokens, 1 generated tokens; copies min(cap, count) into buf, *n = count */
int gb_scheduler_request_tokens(gb_scheduler* s, uint64_t request_id, int which, int32_t* buf,
                                int64_t cap, int64_t* n);

/* ---- op-level entry points (device pointers) ------------------------------------------------
 * The kernels behind the executor, exposed for operator tests and the operator sweep.  They
 * replace the CUDA ops of ggml-cuda the reference dispatches on this path.  Layouts:
 *   Q8_0/Q4_0 weight W[N][K] in the engine's split-row layout written by gb_repack_blocks:
 *   `wq` = N rows, each the K/32 blocks' quants in block order (Q4_0: 16 bytes per block; Q8_0:
 *   bytes 0-15 of every block, then bytes 16-31 of every block), then the fp16 scales in groups
 *   of 64 blocks (within a group: block 32i + l at position 2l + i), zero-padded to whole groups:
 *   gb_weight_row_bytes(type, K) per row;
 *   Q8_0 activations X[M][K]: `xq` int8 [M][K], `xd` fp32 [M][K/32]. */

/* Bytes of one weight row in the split-row layout (Q8_0 = 8, Q4_0 = 2). */
int64_t gb_weight_row_bytes(int type, int64_t K);
/* Element offset of K (or V) row (h, t), head_dim hd, of one sequence in a layer's f16 cache,
 * as every attention kernel addresses it: the contiguous window [H][ctx][hd] when pages is NULL;
 * else the layer's page pool [page][H][1 << page_shift][hd] with `pages` the sequence's page
 * list (pages[i] holds positions [i << page_shift, (i + 1) << page_shift)).  Host arithmetic
 * only; -1 for negative arguments or a shift outside 0..16. */
int64_t gb_kv_row_offset(const int32_t* pages, int page_shift, int64_t H, int64_t ctx, int64_t h,
                         int64_t t, int64_t hd);
/* GGUF block rows (34-byte Q8_0 / 18-byte Q4_0 blocks) -> wq (split-row layout, padding
 * zeroed).  gguf is device memory.  Replaces the weight upload of ggml_backend_tensor_set
 * (executor.cpp:414-429). */
int gb_repack_blocks(const void* gguf, int type, int64_t N, int64_t K, void* wq, void* stream);
/* Activation quantization, quantize_row_q8_0 (ggml-cpu/arch/x86/quants.c:302-392 semantics;
 * the ggml-cuda twin is quantize_q8_1, quantize.cu:54-99).  x rows x_stride floats apart. */
int gb_quantize_q8_0(const float* x, int64_t x_stride, int64_t M, int64_t K, int8_t* xq,
                     float* xd, void* stream);
/* MUL_MAT Y[M][N] = X W^T (+bias[N]) (+residual[M][N]) — ggml_cuda_mul_mat
 * (ggml-cuda.cu:1812-1866: mul_mat_vec_q mmvq.cu:508 for M <= 8, mul_mat_q mmq.cuh:948
 * above; here M > 16 runs on tcgen05, gb_gemm_tc, when K % 128 == 0).  Block int32 dots are exact; block terms accumulate in fp32 (generic block formula of
 * ggml-cpu/quants.c:225-256, :451-477). */
int gb_mul_mat_q(int type, const void* wq, int64_t N, int64_t K,
                 const int8_t* xq, const float* xd, int64_t M, float* y, const float* bias,
                 const float* residual, void* stream);
/* The same MUL_MAT on the 5th-generation tensor cores, any M, K a multiple of 128 (mul_mat_q
 * mmq.cuh:948 is the reference's large-M kernel): operands brought in by the TMA engine, one
 * tcgen05.mma kind::i8 per 32-element block into tensor memory, the block scales applied by
 * epilogue warps; block dots exact, block terms summed in fp32 in block order.  gb_mul_mat_q
 * runs it for M > 16 whenever K % 128 == 0; xq, xd and wq 16-byte aligned.
 * gb_gemm_tc_error returns its sticky error word: 0 while every bounded
 * wait inside it completed, non-zero after one ran out (that launch left its tile unwritten),
 * -1 if the word cannot be read. */
int gb_gemm_tc(int type, const void* wq, int64_t N, int64_t K, const int8_t* xq, const float* xd,
               int64_t M, float* y, const float* bias, const float* residual, void* stream);
int gb_gemm_tc_error(void);
int gb_gemv_error(void);
/* Decode matmul with fused prologue / epilogue, same arithmetic as gb_mul_mat_q.  Input: Q8_0
 * rows (xq, xd; xq 16-byte aligned; any M: the GEMV for 1-2 rows, the tensor-core decode kernel
 * for 3-16, the block GEMM above) or, when xf != NULL, f32 rows [M][K], M <= 4, put through
 * RMS_NORM(eps) (* gamma) and Q8_0 quantization first (the GEMV).  Output: y [M][N] (+bias, +residual); or with swiglu != 0 the
 * SwiGLU of row pairs (n, n+N/2) as f32 y [M][N/2] and/or Q8_0 yq [M][N/2], yd [M][N/64].
 * A single row without Q8_0 output runs on the bulk-copy GEMV (weight rows streamed into
 * per-warp shared-memory rings).  Replaces the ggml-cuda sequence rms_norm_f32 ->
 * quantize_q8_1 -> mul_mat_vec_q -> unary_gated_op_kernel (norm.cu:77, quantize.cu:54,
 * mmvq.cu:508, unary.cu:263).  gb_gemv_error: the sticky error word of that single-row kernel,
 * 0 while every bounded wait in it completed, non-zero after one ran out (that launch left its
 * rows unwritten), -1 if the word cannot be read. */
int gb_gemv(int type, const void* wq, int64_t N, int64_t K, int64_t M,
            const int8_t* xq, const float* xd, const float* xf, float eps, const float* gamma,
            int swiglu, float* y, int8_t* yq, float* yd, const float* bias,
            const float* residual, void* stream);
/* Decode attention for one new token, fused with its RoPE and KV-cache write: qkv is the f32
 * projection row [(Hq + 2 Hkv) * hd] (q heads, then k, then v); the new k (rotated) and v rows go
 * to cache row kv_pos; o [Hq][hd] f32 and/or oq/od Q8_0.  table / n_pos / n_dims as
 * gb_rope_neox (n_dims 0: no rotation).  work: gb_attn_decode_workspace_bytes() of device
 * scratch for the split partials; with head_dim 64 / 128 and caches up to a few thousand
 * positions the kernel runs as one launch whose thread-block clusters merge their partials in
 * distributed shared memory and does not read it.  Replaces rope_neox + k_set_rows +
 * flash_attn_ext_vec (rope.cu:116, set-rows.cu:114, fattn-vec.cuh:21). */
size_t gb_attn_decode_workspace_bytes(int64_t Hq, int64_t Hkv, int64_t hd, int64_t ctx);
int gb_attn_decode(const float* qkv, int64_t Hq, int64_t Hkv, int64_t hd, void* k, void* v,
                   int64_t ctx, int64_t kv_pos, int n_dims, float freq_base, const void* table,
                   int64_t n_pos, float scale, float* o, int8_t* oq, float* od, void* work,
                   void* stream);
/* gb_attn_decode without the work argument, for callers that cannot allocate device memory.
 * No counterpart in the reference (which sizes this scratch from its own CUDA memory pool).
 * Allocates nothing: the split scratch is one fixed 4 MiB device array per device
 * (gb_attn_decode_noalloc_max_bytes()), holding gb_attn_decode_workspace_bytes(Hq, Hkv, hd, ctx)
 * bytes; larger shapes are rejected with an error before anything runs.  Its contents need no
 * initial value (every partial is written before it is read).  The first call on a device looks
 * up the array's address with that device current (setup): make it before any stream capture on
 * that device.  The looked-up address is kept for the life of the process's context on that
 * device: after cudaDeviceReset (or anything else that ends the context) the address is stale,
 * so a process that resets a device must not call this entry point again; start a new process
 * instead.  All calls on one device share the array, so two calls whose kernels can overlap
 * (different streams without ordering, or different host threads) race on it; order them on one
 * stream.  Same results as gb_attn_decode. */
size_t gb_attn_decode_noalloc_max_bytes(void);
int gb_attn_decode_noalloc(const float* qkv, int64_t Hq, int64_t Hkv, int64_t hd, void* k,
                           void* v, int64_t ctx, int64_t kv_pos, int n_dims, float freq_base,
                           const void* table, int64_t n_pos, float scale, float* o, int8_t* oq,
                           float* od, void* stream);
/* GET_ROWS with dequantization — k_get_rows (getrows.cu:6, get_rows_cuda_q :160) */
int gb_get_rows(int type, const void* wq, int64_t N, int64_t K,
                const int32_t* ids, int64_t n, float* out, void* stream);
/* RMS_NORM (+gamma), optional fused Q8_0 output — rms_norm_f32 (norm.cu:77-156) */
int gb_rms_norm(const float* x, int64_t M, int64_t D, float eps, const float* gamma, float* y,
                int8_t* yq, float* yd, void* stream);
/* NORM (LayerNorm, GPT-2 blocks), optional gamma / beta and fused Q8_0 output — norm_f32
 * (ggml-cuda/norm.cu:5, norm_f32_cuda :280); arithmetic of the CPU path
 * ggml_compute_forward_norm_f32 (ggml-cpu/ops.cpp:3762) */
int gb_layer_norm(const float* x, int64_t M, int64_t D, float eps, const float* gamma,
                  const float* beta, float* y, int8_t* yq, float* yd, void* stream);
/* bias + tanh-GELU of the GPT-2 MLP, optional fused Q8_0 output — ggmlc's CPU custom op
 * ggmlc_compute_forward_bias_gelu (runtime/src/stdlib_kernels.cpp:29, fast_gelu_f32 :9) and
 * the ADD + GELU pair it stands for on CUDA (ggml-cuda/unary.cu:20 op_gelu) */
int gb_bias_gelu(const float* x, const float* bias, int64_t M, int64_t F, float* y, int8_t* yq,
                 float* yd, void* stream);
/* SWIGLU over [gate(F) ; up(F)] rows, optional fused Q8_0 output — unary.cu:263-337 */
int gb_swiglu(const float* x, int64_t M, int64_t F, float* y, int8_t* yq, float* yd,
              void* stream);
/* Host helper: fill (cos, sin) pairs [n_pos][n_dims/2] exactly as the CPU RoPE cache does
 * (ggml-cpu/ops.cpp:5910-5923: fp32 theta recurrence, libm cosf/sinf).  Returns theta_scale. */
float gb_rope_table_fill(float* host_out, int64_t n_pos, int n_dims, float freq_base);
/* NEOX RoPE of x[s][H][hd] (f32) at positions pos[s] -> y — rope_neox (rope.cu:116-183).
 * table: device copy of gb_rope_table_fill output for n_pos positions, or NULL (cos/sin are
 * then evaluated on the device). */
int gb_rope_neox(const float* x, int64_t hd, int64_t H, int64_t s, const int32_t* pos,
                 int n_dims, float freq_base, const void* table, int64_t n_pos, float* y,
                 void* stream);
/* Attention of q[s][Hq][hd] (f32) over f16 caches k, v [Hkv][ctx][hd]; query i sees cache
 * rows 0..kv_pos+i; output o[s][Hq][hd] — flash_attn_ext_vec / _f16 (fattn-vec.cuh:21,
 * fattn-mma-f16.cuh:1705).  work: gb_attention_workspace_bytes() of device scratch. */
size_t gb_attention_workspace_bytes(int64_t s, int64_t Hq, int64_t hd, int64_t ctx);
int gb_attention(const float* q, const void* k, const void* v, int64_t hd, int64_t s,
                 int64_t Hq, int64_t Hkv, int64_t ctx, int64_t kv_pos, float scale, float* o,
                 void* work, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GGMLC_B200_H */
