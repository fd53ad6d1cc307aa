// Host page allocator of the KV pool: the "page allocate / free / compact" part of
// the scheduler. Policy: the lowest free page id is handed out first, so block
// tables are a deterministic function of the open/append/close order (the CPU
// oracle restates the same policy and checks block tables for byte identity).
// Compaction moves the highest live page into the lowest free id until the live
// pages occupy [0, n_live), which shrinks the pool's high-water mark.
#pragma once

#include <cstdint>
#include <vector>

namespace fa {

class PageAllocator {
public:
    void init(int n_pages) {
        n_pages_ = n_pages;
        n_free_ = n_pages;
        bits_.assign((n_pages + 63) / 64, ~0ull);
        if (n_pages % 64) bits_.back() = (1ull << (n_pages % 64)) - 1;
        hint_ = 0;
    }
    int n_pages() const { return n_pages_; }
    int n_free() const { return n_free_; }

    // Returns a page id or -1 when the pool is exhausted.
    int alloc() {
        for (size_t w = hint_; w < bits_.size(); ++w) {
            if (bits_[w]) {
                const int b = __builtin_ctzll(bits_[w]);
                bits_[w] &= bits_[w] - 1;
                --n_free_;
                hint_ = w;
                return (int)(w * 64 + b);
            }
        }
        hint_ = bits_.size();
        return -1;
    }
    bool is_free(int p) const { return (bits_[p / 64] >> (p % 64)) & 1ull; }
    // Returns false on a page outside the pool or already free.
    bool release(int p) {
        if (p < 0 || p >= n_pages_ || is_free(p)) return false;
        bits_[p / 64] |= 1ull << (p % 64);
        ++n_free_;
        if ((size_t)(p / 64) < hint_) hint_ = p / 64;
        return true;
    }
    // Compaction plan applied to the bitmap: returns (src, dst) moves in order.
    void compact(std::vector<int>& src, std::vector<int>& dst) {
        src.clear();
        dst.clear();
        int lo = 0, hi = n_pages_ - 1;
        while (true) {
            while (lo < n_pages_ && !is_free(lo)) ++lo;
            while (hi >= 0 && is_free(hi)) --hi;
            if (lo >= n_pages_ || hi < 0 || lo > hi) break;
            src.push_back(hi);
            dst.push_back(lo);
            bits_[lo / 64] &= ~(1ull << (lo % 64));
            bits_[hi / 64] |= 1ull << (hi % 64);
        }
        hint_ = 0;
    }

private:
    std::vector<uint64_t> bits_;   // 1 = free
    int n_pages_ = 0;
    int n_free_ = 0;
    size_t hint_ = 0;              // no free page below word hint_
};

}  // namespace fa
