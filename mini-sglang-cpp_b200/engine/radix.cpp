// radix.cpp -- prefix cache over KV pages (host side).
//
// RadixCache (src/cache/kvcache.cpp:40-115, include/minisgl/cache/kvcache.h:35-72) maps token
// prefixes to the KV pages that already hold them, so a new request reuses a cached prefix
// (Scheduler::schedule_next_batch, src/scheduler/scheduler.cpp:45-49). This tree keeps that role
// and interface shape (match / insert / evict) with the reference's defects fixed:
//  * page granularity: a node holds a run of whole pages (page_size tokens each) and a match
//    counts whole pages only -- a KV page is shared whole or not at all (the reference matches
//    token by token with one page per token and an off-by-one in its page loop);
//  * insert walks and extends the tree (the reference attaches one node under the root,
//    replacing any sibling with the same first token), splitting a node where a new sequence
//    diverges at a page boundary inside it;
//  * reference counts: a running request locks the path of its matched node, and only unlocked
//    leaves are evicted (the reference evicts root children only and never counts references);
//  * eviction is page by page: the least recently used unlocked leaf (ties: the lower last page
//    id) gives up its last page; pages return to the caller, which owns the free list.
// Handles are node ids (0 = the root); a node keeps its id when a split inserts a node above it.
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "msgl_engine.h"

namespace msgl {
int set_error(int code, const char* msg);
}

struct msgl_radix {
    struct Node {
        int64_t id = 0;
        std::vector<int32_t> key;    // tokens: pages.size() * page_size
        std::vector<int32_t> pages;  // KV pages holding `key`
        Node* parent = nullptr;
        std::map<std::vector<int32_t>, Node*> children;  // keyed by the child's first page of tokens
        int64_t ref = 0;
        uint64_t time = 0;
    };
    int P = 16;
    uint64_t clock = 0;
    int64_t next_id = 1;
    Node root;
    std::unordered_map<int64_t, std::unique_ptr<Node>> nodes;

    std::vector<int32_t> chunk(const int32_t* t, int64_t off) const {
        return std::vector<int32_t>(t + off, t + off + P);
    }
    Node* node_of(int64_t id) {
        if (id == 0) return &root;
        auto it = nodes.find(id);
        if (it == nodes.end()) throw std::runtime_error("radix: unknown node handle");
        return it->second.get();
    }
    // splits `c` after its first `j` pages (0 < j < pages): a new node above `c` takes them
    Node* split(Node* c, size_t j) {
        auto mid = std::make_unique<Node>();
        Node* m = mid.get();
        m->id = next_id++;
        m->key.assign(c->key.begin(), c->key.begin() + static_cast<int64_t>(j) * P);
        m->pages.assign(c->pages.begin(), c->pages.begin() + static_cast<int64_t>(j));
        m->parent = c->parent;
        m->ref = c->ref;    // every lock through c passes through m
        m->time = c->time;
        c->parent->children[chunk(c->key.data(), 0)] = m;
        c->key.erase(c->key.begin(), c->key.begin() + static_cast<int64_t>(j) * P);
        c->pages.erase(c->pages.begin(), c->pages.begin() + static_cast<int64_t>(j));
        c->parent = m;
        m->children[chunk(c->key.data(), 0)] = c;
        nodes[m->id] = std::move(mid);
        return m;
    }
    // walks the longest cached page-aligned prefix of t[0, n); returns the node where it ends
    // (split there if it ends inside a node) and appends its pages to `pages`
    Node* walk(const int32_t* t, int64_t n, int64_t& matched, std::vector<int32_t>* pages) {
        Node* node = &root;
        matched = 0;
        while (matched + P <= n) {
            auto it = node->children.find(chunk(t, matched));
            if (it == node->children.end()) break;
            Node* c = it->second;
            size_t j = 0;
            while (j < c->pages.size() && matched + P <= n &&
                   std::equal(c->key.begin() + static_cast<int64_t>(j) * P,
                              c->key.begin() + static_cast<int64_t>(j + 1) * P, t + matched)) {
                if (pages) pages->push_back(c->pages[j]);
                matched += P;
                ++j;
            }
            if (j < c->pages.size()) return split(c, j);  // j >= 1: the first page matched
            node = c;
        }
        return node;
    }
    void touch(Node* n) {
        const uint64_t now = ++clock;
        for (; n && n != &root; n = n->parent) n->time = now;
    }
};

namespace {
template <typename F>
int guarded(F&& f) {
    try {
        f();
        return MSGL_OK;
    } catch (const std::bad_alloc&) {
        return msgl::set_error(MSGL_ERR_WORKSPACE, "radix: out of host memory");
    } catch (const std::exception& e) {
        return msgl::set_error(MSGL_ERR_INVALID_ARG, e.what());
    }
}
}  // namespace

extern "C" {

int msgl_radix_create(int page_size, msgl_radix** out) {
    if (!out || page_size <= 0) return msgl::set_error(MSGL_ERR_INVALID_ARG, "radix_create: bad args");
    *out = nullptr;
    return guarded([&] {
        auto* r = new msgl_radix();
        r->P = page_size;
        *out = r;
    });
}

int msgl_radix_destroy(msgl_radix* r) {
    delete r;
    return MSGL_OK;
}

int msgl_radix_match(msgl_radix* r, const int32_t* tokens, int num_tokens, int32_t* pages_out,
                     int max_pages, int* matched_tokens, int64_t* node) {
    if (!r || num_tokens < 0 || (num_tokens > 0 && !tokens) || !matched_tokens)
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "radix_match: bad args");
    return guarded([&] {
        std::vector<int32_t> pages;
        int64_t m = 0;
        msgl_radix::Node* n = r->walk(tokens, num_tokens, m, &pages);
        if (static_cast<int64_t>(pages.size()) > max_pages || (!pages.empty() && !pages_out))
            throw std::runtime_error("radix_match: pages_out holds fewer pages than the match");
        r->touch(n);
        for (size_t i = 0; i < pages.size(); ++i) pages_out[i] = pages[i];
        *matched_tokens = static_cast<int>(m);
        if (node) *node = n->id;
    });
}

int msgl_radix_insert(msgl_radix* r, const int32_t* tokens, int num_tokens, const int32_t* pages,
                      int* present_tokens, int32_t* dup_pages_out, int* num_dup, int64_t* node) {
    if (!r || num_tokens < 0 || (num_tokens >= r->P && (!tokens || !pages)))
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "radix_insert: bad args");
    return guarded([&] {
        const int64_t full = num_tokens - num_tokens % r->P;
        std::vector<int32_t> have;
        int64_t m = 0;
        msgl_radix::Node* n = r->walk(tokens, full, m, &have);
        // the caller's pages for the part already cached, where they differ from the tree's
        int nd = 0;
        for (size_t i = 0; i < have.size(); ++i)
            if (pages[i] != have[i]) {
                if (dup_pages_out) dup_pages_out[nd] = pages[i];
                ++nd;
            }
        if (m < full) {
            auto leaf = std::make_unique<msgl_radix::Node>();
            msgl_radix::Node* l = leaf.get();
            l->id = r->next_id++;
            l->key.assign(tokens + m, tokens + full);
            l->pages.assign(pages + m / r->P, pages + full / r->P);
            l->parent = n;
            n->children[r->chunk(l->key.data(), 0)] = l;
            r->nodes[l->id] = std::move(leaf);
            n = l;
        }
        r->touch(n);
        if (present_tokens) *present_tokens = static_cast<int>(m);
        if (num_dup) *num_dup = nd;
        if (node) *node = n->id;
    });
}

int msgl_radix_lock(msgl_radix* r, int64_t node, int delta) {
    if (!r || (delta != 1 && delta != -1)) return msgl::set_error(MSGL_ERR_INVALID_ARG, "radix_lock: bad args");
    return guarded([&] {
        msgl_radix::Node* n = r->node_of(node);
        for (msgl_radix::Node* p = n; p != &r->root; p = p->parent)
            if (delta < 0 && p->ref == 0) throw std::runtime_error("radix_lock: unlock of an unlocked node");
        for (msgl_radix::Node* p = n; p != &r->root; p = p->parent) p->ref += delta;
    });
}

int msgl_radix_evict(msgl_radix* r, int num_pages, int32_t* freed_out, int* num_freed) {
    if (!r || num_pages < 0 || (num_pages > 0 && !freed_out) || !num_freed)
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "radix_evict: bad args");
    return guarded([&] {
        int freed = 0;
        while (freed < num_pages) {
            msgl_radix::Node* best = nullptr;
            for (auto& kv : r->nodes) {
                msgl_radix::Node* c = kv.second.get();
                if (!c->children.empty() || c->ref > 0) continue;
                if (!best || c->time < best->time ||
                    (c->time == best->time && c->pages.back() < best->pages.back()))
                    best = c;
            }
            if (!best) break;  // everything left is locked or an inner node
            freed_out[freed++] = best->pages.back();
            best->pages.pop_back();
            best->key.resize(best->key.size() - r->P);
            if (best->pages.empty()) {
                // its key in the parent's map was its first page, now gone: find it by pointer
                for (auto it = best->parent->children.begin(); it != best->parent->children.end(); ++it)
                    if (it->second == best) {
                        best->parent->children.erase(it);
                        break;
                    }
                r->nodes.erase(best->id);
            }
        }
        *num_freed = freed;
    });
}

int msgl_radix_size(const msgl_radix* r, int* cached_pages, int* evictable_pages) {
    if (!r) return msgl::set_error(MSGL_ERR_INVALID_ARG, "radix_size: null");
    int64_t total = 0, unlocked = 0;
    for (auto& kv : r->nodes) {
        total += static_cast<int64_t>(kv.second->pages.size());
        if (kv.second->ref == 0) unlocked += static_cast<int64_t>(kv.second->pages.size());
    }
    if (cached_pages) *cached_pages = static_cast<int>(total);
    if (evictable_pages) *evictable_pages = static_cast<int>(unlocked);
    return MSGL_OK;
}

}  // extern "C"
