#include "radix.h"

#include <cstring>
#include <functional>

#include "common.h"

namespace gb {

PrefixTree::PrefixTree(int64_t tokens_per_page)
    : T_(tokens_per_page), root_(std::make_unique<Node>()) {
    GB_CHECK(T_ >= 1, "prefix tree: tokens_per_page must be positive");
}

PrefixTree::~PrefixTree() = default;

uint64_t PrefixTree::chunk_hash(const int32_t* tokens, size_t count) {
    uint64_t h = 14695981039346656037ULL;  // FNV-1a 64-bit offset basis
    for (size_t i = 0; i < count; ++i) {
        const uint32_t v = (uint32_t)tokens[i];
        for (int b = 0; b < 4; ++b) {
            h ^= (v >> (8 * b)) & 0xFFu;
            h *= 1099511628211ULL;  // FNV-1a 64-bit prime
        }
    }
    return h;
}

PrefixTree::Node* PrefixTree::child(Node* n, const int32_t* chunk) const {
    auto it = n->children.find(chunk_hash(chunk, (size_t)T_));
    if (it == n->children.end()) return nullptr;
    Node* c = it->second.get();
    // a hash hit counts only if the tokens agree
    if (std::memcmp(c->chunk.data(), chunk, sizeof(int32_t) * (size_t)T_) != 0) return nullptr;
    return c;
}

PrefixTree::Node* PrefixTree::attach(Node* parent, const int32_t* chunk, int64_t page) {
    auto n = std::make_unique<Node>();
    n->chunk.assign(chunk, chunk + T_);
    n->page = page;
    n->parent = parent;
    Node* raw = n.get();
    parent->children.emplace(chunk_hash(chunk, (size_t)T_), std::move(n));  // key checked free
    ++n_pages_;
    return raw;
}

PrefixMatch PrefixTree::match(const std::vector<int32_t>& tokens) {
    PrefixMatch m;
    const int64_t full = (int64_t)tokens.size() / T_;
    Node* cur = root_.get();
    for (int64_t p = 0; p < full; ++p) {
        Node* c = child(cur, tokens.data() + p * T_);
        if (!c) break;
        c->tick = ++tick_;
        m.pages.push_back(c->page);
        cur = c;
    }
    m.matched_pages = (int64_t)m.pages.size();
    m.matched_tokens = m.matched_pages * T_;
    return m;
}

int64_t PrefixTree::evict_lru() {
    Node* best = nullptr;
    std::function<void(Node*)> walk = [&](Node* n) {
        for (auto& [h, c] : n->children) {
            if (c->children.empty()) {
                if (!c->pinned && (!best || c->tick < best->tick)) best = c.get();
            } else {
                walk(c.get());
            }
        }
    };
    walk(root_.get());
    if (!best) return -1;
    const int64_t page = best->page;
    Node* parent = best->parent;
    parent->children.erase(chunk_hash(best->chunk.data(), (size_t)T_));
    --n_pages_;
    return page;
}

void PrefixTree::reset() {
    root_ = std::make_unique<Node>();
    n_pages_ = 0;
    tick_ = 0;
}

}  // namespace gb
