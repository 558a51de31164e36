// Prefix cache index: a trie over whole pages of prompt tokens (tokens_per_page tokens per
// edge), each node naming the page of KV-cache rows computed for its chunk.  The counterpart of
// the reference's PagedRadixTree (runtime/include/ggmlc/radix_tree.h,
// runtime/src/radix_tree.cpp:7-220): chunks are keyed by a 64-bit FNV-1a hash of their tokens'
// bytes and verified token by token, matching walks whole pages from the root, and pages are
// reclaimed least-recently-used first, leaves only.
//
// The tree only indexes: a page id here is a page of the executor's paged KV pool, which the
// scheduler holds a reference to for as long as the node exists and maps into a sequence's page
// table on a hit.
#pragma once

#include <cstdint>
#include <memory>
#include <unordered_map>
#include <vector>

namespace gb {

struct PrefixMatch {
    int64_t matched_pages = 0;
    int64_t matched_tokens = 0;
    std::vector<int64_t> pages;  // pool page of each matched chunk, root first
};

class PrefixTree {
public:
    explicit PrefixTree(int64_t tokens_per_page);
    ~PrefixTree();

    // 64-bit FNV-1a over the four little-endian bytes of each token (radix_tree.cpp:7-22)
    static uint64_t chunk_hash(const int32_t* tokens, size_t count);

    int64_t tokens_per_page() const { return T_; }
    // the longest run of whole pages of `tokens` present in the tree; marks them used
    PrefixMatch match(const std::vector<int32_t>& tokens);
    // Attach pages [first, first + n) of `tokens` below its first `first` pages, which must be in
    // the tree (else nothing is attached).  page_of(i) gives the pool page for chunk first + i
    // and is called only for chunks not yet present; it may call evict_lru(), which never takes
    // a node of this path.  Returns the number of chunks newly attached.
    template <class F>
    int64_t insert(const std::vector<int32_t>& tokens, int64_t first, int64_t n, F&& page_of);
    // Remove the least recently used leaf (not on a path being inserted); its page, or -1 when
    // every node is in use.
    int64_t evict_lru();
    int64_t total_pages() const { return n_pages_; }
    int64_t total_nodes() const { return n_pages_ + 1; }  // + the root
    void reset();

private:
    struct Node {
        std::vector<int32_t> chunk;
        int64_t page = -1;
        uint64_t tick = 0;
        bool pinned = false;
        Node* parent = nullptr;
        std::unordered_map<uint64_t, std::unique_ptr<Node>> children;
    };
    Node* child(Node* n, const int32_t* chunk) const;
    Node* attach(Node* parent, const int32_t* chunk, int64_t page);

    int64_t T_;
    uint64_t tick_ = 0;
    int64_t n_pages_ = 0;
    std::unique_ptr<Node> root_;
};

template <class F>
int64_t PrefixTree::insert(const std::vector<int32_t>& tokens, int64_t first, int64_t n,
                           F&& page_of) {
    if (first < 0 || n <= 0 || (first + n) * T_ > (int64_t)tokens.size()) return 0;
    std::vector<Node*> path;
    Node* cur = root_.get();
    for (int64_t p = 0; p < first; ++p) {
        cur = child(cur, tokens.data() + p * T_);
        if (!cur) {
            for (Node* q : path) q->pinned = false;
            return 0;
        }
        cur->pinned = true;
        path.push_back(cur);
    }
    int64_t added = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int32_t* chunk = tokens.data() + (first + i) * T_;
        Node* nx = child(cur, chunk);
        if (!nx) {
            if (cur->children.count(chunk_hash(chunk, (size_t)T_))) break;  // hash taken
            const int64_t page = page_of(i);
            if (page < 0) break;  // no page to hold it
            nx = attach(cur, chunk, page);
            ++added;
        }
        nx->tick = ++tick_;
        nx->pinned = true;
        path.push_back(nx);
        cur = nx;
    }
    for (Node* q : path) q->pinned = false;
    return added;
}

}  // namespace gb
