// page_table.h -- the host side of the paged KV pool: which physical page of
// 16 positions holds each sequence's logical page, and which pages are free.
//
// The reference keeps one contiguous [capacity, n_embd] block per layer for its
// single sequence (src/kv_cache.c:150-190). A batch pool here holds n_pages
// physical pages per layer and assigns them to sequences as their contexts
// grow: map(seq, length) gives seq the pages that cover positions
// [0, length), release(seq) returns them for reuse. The kernels address every
// position through the device copy of the table (PagedKV::row); device_view()
// writes that copy with unmapped entries pointing at a scratch page (index
// n_pages, one past the assignable ones), so a stale entry can never send a
// kernel outside the pool.
//
// Pure host C++ (no CUDA), so the allocator is tested on its own.
#pragma once

#include <cstddef>
#include <vector>

namespace tie {

class PageTable {
public:
    static constexpr int kRows = 16;   // positions per page

    PageTable() = default;
    // n_seq sequences of up to `capacity` positions over n_pages physical pages
    PageTable(int n_seq, int capacity, int n_pages)
        : n_seq_(n_seq), pages_per_seq_((capacity + kRows - 1) / kRows), n_pages_(n_pages),
          table_((size_t)n_seq * pages_per_seq_, -1), mapped_((size_t)n_seq, 0) {
        free_.reserve((size_t)n_pages);
        for (int p = n_pages - 1; p >= 0; --p) free_.push_back(p);   // page 0 is handed out first
    }

    int n_seq() const { return n_seq_; }
    int pages_per_seq() const { return pages_per_seq_; }
    int n_pages() const { return n_pages_; }
    int scratch_page() const { return n_pages_; }
    int free_pages() const { return (int)free_.size(); }
    int mapped_pages(int seq) const { return mapped_[(size_t)seq]; }
    // the physical page of a sequence's logical page, or -1 when unmapped
    int page(int seq, int logical) const { return table_[(size_t)seq * pages_per_seq_ + logical]; }
    bool dirty() const { return dirty_; }

    // Maps pages so that seq covers positions [0, length). Returns false, with
    // nothing changed, when length exceeds the capacity or too few pages are free.
    bool map(int seq, int length) {
        if (seq < 0 || seq >= n_seq_ || length < 0) return false;
        const int need = (length + kRows - 1) / kRows;
        if (need > pages_per_seq_) return false;
        int& have = mapped_[(size_t)seq];
        if (need <= have) return true;
        if (need - have > (int)free_.size()) return false;
        for (; have < need; ++have) {
            table_[(size_t)seq * pages_per_seq_ + have] = free_.back();
            free_.pop_back();
        }
        dirty_ = true;
        return true;
    }

    // Returns every page of seq to the free list (last mapped first).
    void release(int seq) {
        if (seq < 0 || seq >= n_seq_) return;
        int& have = mapped_[(size_t)seq];
        for (; have > 0; --have) {
            int& e = table_[(size_t)seq * pages_per_seq_ + have - 1];
            free_.push_back(e);
            e = -1;
            dirty_ = true;
        }
    }

    // The table as the kernels read it: unmapped entries point at the scratch page.
    const std::vector<int>& device_view() {
        view_.resize(table_.size());
        for (size_t i = 0; i < table_.size(); ++i) view_[i] = table_[i] < 0 ? n_pages_ : table_[i];
        dirty_ = false;
        return view_;
    }

private:
    int n_seq_ = 0, pages_per_seq_ = 0, n_pages_ = 0;
    std::vector<int> table_;    // [n_seq][pages_per_seq], -1 = unmapped
    std::vector<int> mapped_;   // pages mapped per sequence (always a prefix)
    std::vector<int> free_;     // stack of free physical pages
    std::vector<int> view_;
    bool dirty_ = true;
};

}  // namespace tie
