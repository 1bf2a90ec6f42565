// kv_cache.h -- the paged fp16 KV cache allocator.
//
// The reference has no pages: it sizes one contiguous fp32 region
// [layer][K|V][kvHead][maxPos][headDim] plus a 2-word argmax tail
// (Opure_Graph.h:81-84, Opure_Graph.cpp:396-400, Opure_VoxelEngine.cpp:143-148), so every
// sequence costs max_position_embeddings of cache up front. Here each layer owns a pool of
// fixed-size pages laid out [page][K|V][n_kv][page_size][head_dim] (fp16); a page id is
// valid in every layer's pool, and each sequence slot has a row of the int32 page table
// mapping logical page -> physical page. Pages come from a free list (optionally shuffled
// with a seeded Fisher-Yates permutation, so tests exercise non-contiguous tables);
// truncation (speculative rollback) and release return pages to it.
//
// Sliding window (ring > 0): a sequence holds at most `ring` pages, used as a ring (position
// p in table entry (p / page_size) % ring, opure_kv_layout.ring); when it moves past them it
// overwrites its own oldest page in place instead of mapping a new one. This replaces the
// reference's eviction, which shifts the whole cache by one position with a memmove
// dispatch per layer (EvictOldestKV, Opure_VoxelEngine.cpp:721-763; Opure_Memmove.usf).
#pragma once

#include <cstdint>
#include <vector>

#include "graph.h"
#include "opure_cuda.h"

namespace opure::kv {

class PagedKvCache {
public:
    PagedKvCache() = default;
    ~PagedKvCache();
    PagedKvCache(const PagedKvCache &) = delete;
    PagedKvCache &operator=(const PagedKvCache &) = delete;

    void Create(opure_ctx *ctx, const graph::ModelConfig &cfg, uint32_t page_size, uint32_t n_pages,
                uint32_t max_seqs, uint32_t max_pages_per_seq, uint64_t shuffle_seed, uint32_t ring = 0);
    void Destroy();

    // Maps pages for positions [0, tokens) of `seq` (with a window: at most `ring` pages,
    // which then hold any position). Returns false (nothing changed) when the free list or
    // the table row is too short.
    bool Reserve(uint32_t seq, uint32_t tokens);
    // Whether position `pos` of `seq` has a mapped page.
    bool Covers(uint32_t seq, uint32_t pos) const;
    uint32_t Ring() const { return ring_; }
    void Truncate(uint32_t seq, uint32_t tokens);  // unmap pages wholly past `tokens`
    void Release(uint32_t seq);
    void SyncTable();                              // upload the table when it changed

    opure_kv_layout Layout(uint32_t layer) const;
    uint16_t *Pool(uint32_t layer) const;
    const int32_t *DeviceTable() const { return dTable_; }
    uint32_t PageSize() const { return pageSize_; }
    uint32_t MaxPages() const { return maxPages_; }
    uint32_t NumPages() const { return nPages_; }
    uint32_t FreePages() const { return uint32_t(free_.size()); }
    uint32_t MappedPages(uint32_t seq) const;
    uint64_t PoolBytesPerLayer() const { return poolBytes_; }
    const std::vector<int32_t> &HostTable() const { return table_; }

private:
    opure_ctx *ctx_ = nullptr;
    uint32_t layers_ = 0, nKv_ = 0, headDim_ = 0;
    uint32_t pageSize_ = 0, nPages_ = 0, maxSeqs_ = 0, maxPages_ = 0, ring_ = 0;
    uint64_t poolBytes_ = 0;
    void *pools_ = nullptr;            // layers_ * poolBytes_
    int32_t *dTable_ = nullptr;        // [maxSeqs_][maxPages_]
    std::vector<int32_t> table_;       // host mirror, -1 = unmapped
    std::vector<uint32_t> mapped_;     // pages mapped per sequence
    std::vector<int32_t> free_;        // stack of free page ids
    bool dirty_ = true;
};

}  // namespace opure::kv
