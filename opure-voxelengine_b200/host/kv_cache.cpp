// kv_cache.cpp -- paged KV allocator (see kv_cache.h).
#include "kv_cache.h"

#include <algorithm>

#include "platform.h"
#include "synth.h"

namespace opure::kv {

PagedKvCache::~PagedKvCache() { Destroy(); }

void PagedKvCache::Create(opure_ctx *ctx, const graph::ModelConfig &cfg, uint32_t page_size,
                          uint32_t n_pages, uint32_t max_seqs, uint32_t max_pages_per_seq,
                          uint64_t shuffle_seed, uint32_t ring) {
    Destroy();
    OPURE_CHECK(page_size == 16 || page_size == 32 || page_size == 64 || page_size == 128,
                "KV page size must be 16, 32, 64 or 128 tokens");
    OPURE_CHECK(n_pages > 0 && max_seqs > 0 && max_pages_per_seq > 0, "empty KV cache");
    OPURE_CHECK(ring <= max_pages_per_seq, "KV window longer than a table row");
    ctx_ = ctx;
    layers_ = cfg.numLayers;
    nKv_ = cfg.numKvHeads;
    headDim_ = cfg.HeadDim();
    pageSize_ = page_size;
    nPages_ = n_pages;
    maxSeqs_ = max_seqs;
    maxPages_ = max_pages_per_seq;
    ring_ = ring;
    poolBytes_ = uint64_t(n_pages) * 2 * nKv_ * page_size * headDim_ * 2;
    OPURE_CUDA_CHECK(opure_alloc(ctx_, poolBytes_ * layers_, &pools_));
    OPURE_CUDA_CHECK(opure_fill(ctx_, pools_, 0, poolBytes_ * layers_));
    void *t = nullptr;
    OPURE_CUDA_CHECK(opure_alloc(ctx_, sizeof(int32_t) * size_t(max_seqs) * max_pages_per_seq, &t));
    dTable_ = static_cast<int32_t *>(t);
    table_.assign(size_t(max_seqs) * max_pages_per_seq, -1);
    mapped_.assign(max_seqs, 0);
    std::vector<int32_t> order = shuffle_seed ? synth::Permutation(shuffle_seed, n_pages)
                                              : synth::Permutation(0, 0);
    if (!shuffle_seed) {
        order.resize(n_pages);
        for (uint32_t i = 0; i < n_pages; ++i) order[i] = int32_t(i);
    }
    // Stack: the first page handed out is order[0].
    free_.assign(order.rbegin(), order.rend());
    dirty_ = true;
    SyncTable();
}

void PagedKvCache::Destroy() {
    if (ctx_) {
        if (pools_) opure_free(ctx_, pools_);
        if (dTable_) opure_free(ctx_, dTable_);
    }
    pools_ = nullptr;
    dTable_ = nullptr;
    ctx_ = nullptr;
    table_.clear();
    mapped_.clear();
    free_.clear();
}

bool PagedKvCache::Reserve(uint32_t seq, uint32_t tokens) {
    OPURE_CHECK(seq < maxSeqs_, "KV sequence slot out of range");
    uint32_t need = (tokens + pageSize_ - 1) / pageSize_;
    if (ring_) need = std::min(need, ring_);
    if (need > maxPages_) return false;
    if (need <= mapped_[seq]) return true;
    if (need - mapped_[seq] > free_.size()) return false;
    for (uint32_t lp = mapped_[seq]; lp < need; ++lp) {
        table_[size_t(seq) * maxPages_ + lp] = free_.back();
        free_.pop_back();
    }
    mapped_[seq] = need;
    dirty_ = true;
    return true;
}

void PagedKvCache::Truncate(uint32_t seq, uint32_t tokens) {
    OPURE_CHECK(seq < maxSeqs_, "KV sequence slot out of range");
    const uint32_t keep = (tokens + pageSize_ - 1) / pageSize_;
    while (mapped_[seq] > keep) {
        int32_t &e = table_[size_t(seq) * maxPages_ + --mapped_[seq]];
        free_.push_back(e);
        e = -1;
        dirty_ = true;
    }
}

void PagedKvCache::Release(uint32_t seq) { Truncate(seq, 0); }

uint32_t PagedKvCache::MappedPages(uint32_t seq) const { return seq < maxSeqs_ ? mapped_[seq] : 0; }

bool PagedKvCache::Covers(uint32_t seq, uint32_t pos) const {
    if (seq >= maxSeqs_) return false;
    return (ring_ && mapped_[seq] == ring_) || pos < mapped_[seq] * pageSize_;
}

void PagedKvCache::SyncTable() {
    if (!dirty_ || !ctx_) return;
    OPURE_CUDA_CHECK(opure_h2d(ctx_, dTable_, table_.data(), table_.size() * sizeof(int32_t)));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    dirty_ = false;
}

uint16_t *PagedKvCache::Pool(uint32_t layer) const {
    return reinterpret_cast<uint16_t *>(static_cast<uint8_t *>(pools_) + poolBytes_ * layer);
}

opure_kv_layout PagedKvCache::Layout(uint32_t layer) const {
    opure_kv_layout l{};
    l.pool = Pool(layer);
    l.page_table = dTable_;
    l.n_pages = nPages_;
    l.max_pages = maxPages_;
    l.page_size = pageSize_;
    l.n_kv = nKv_;
    l.head_dim = headDim_;
    l.ring = ring_;
    return l;
}

}  // namespace opure::kv
