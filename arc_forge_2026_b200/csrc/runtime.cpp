// Native serving runtime pieces: the KV page allocator with per-session page lists and reference counts (prefix
// sharing), and the session table the scheduler keeps. Host-only C++; the device sees pages only through the
// int32 block tables the engine uploads.
//
// The reference's scheduler and radix/HiSparse caches live inside its sglang fork (Python); here the page
// bookkeeping that runs every decode step is native so the per-step host cost stays at a few microseconds for
// 128+ sessions.
#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace {

class PageAllocator {
 public:
  PageAllocator(int64_t num_pages, int64_t page_size) : page_size_(page_size), ref_(num_pages, 0) {
    if (num_pages <= 0 || page_size <= 0) throw std::invalid_argument("PageAllocator: sizes must be positive");
    free_.reserve(num_pages);
    for (int64_t p = num_pages - 1; p >= 0; --p) free_.push_back((int32_t)p);  // pop_back hands out page 0 first
  }

  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t num_pages() const { return (int64_t)ref_.size(); }
  int64_t page_size() const { return page_size_; }

  // make session `sid` hold pages for `tokens` tokens; returns the newly allocated pages (appended in order)
  std::vector<int32_t> ensure(int64_t sid, int64_t tokens) {
    auto& pages = sessions_[sid];
    const int64_t need = (tokens + page_size_ - 1) / page_size_;
    std::vector<int32_t> added;
    if ((int64_t)pages.size() >= need) return added;
    const int64_t extra = need - (int64_t)pages.size();
    if (extra > (int64_t)free_.size()) throw std::runtime_error("PageAllocator: out of KV pages");
    for (int64_t i = 0; i < extra; ++i) {
      const int32_t p = free_.back();
      free_.pop_back();
      ref_[p] = 1;
      pages.push_back(p);
      added.push_back(p);
    }
    return added;
  }

  // share the first `tokens` tokens' full pages of `src` with `dst` (prefix reuse; refcounted)
  void fork_prefix(int64_t src, int64_t dst, int64_t tokens) {
    auto it = sessions_.find(src);
    if (it == sessions_.end()) throw std::invalid_argument("fork_prefix: unknown source session");
    auto& d = sessions_[dst];
    if (!d.empty()) throw std::invalid_argument("fork_prefix: destination session already holds pages");
    const int64_t full = std::min<int64_t>(tokens / page_size_, (int64_t)it->second.size());
    for (int64_t i = 0; i < full; ++i) {
      const int32_t p = it->second[i];
      ++ref_[p];
      d.push_back(p);
    }
  }

  void release(int64_t sid) {
    auto it = sessions_.find(sid);
    if (it == sessions_.end()) return;
    for (int32_t p : it->second) {
      if (--ref_[p] == 0) free_.push_back(p);
    }
    sessions_.erase(it);
  }

  std::vector<int32_t> pages(int64_t sid) const {
    auto it = sessions_.find(sid);
    if (it == sessions_.end()) return {};
    return it->second;
  }

  // write session `sid`'s page list into row `row` of an int32 [rows, max_pages] host tensor
  void fill_row(int64_t sid, at::Tensor table, int64_t row) const {
    TORCH_CHECK(table.dtype() == torch::kInt32 && table.dim() == 2 && !table.is_cuda(), "host int32 table");
    auto it = sessions_.find(sid);
    int32_t* r = table.data_ptr<int32_t>() + row * table.size(1);
    const int64_t n = it == sessions_.end() ? 0 : (int64_t)it->second.size();
    TORCH_CHECK(n <= table.size(1), "block table row too short");
    for (int64_t i = 0; i < n; ++i) r[i] = it->second[i];
    for (int64_t i = n; i < table.size(1); ++i) r[i] = 0;
  }

 private:
  int64_t page_size_;
  std::vector<int32_t> free_;
  std::vector<int32_t> ref_;
  std::unordered_map<int64_t, std::vector<int32_t>> sessions_;
};

}  // namespace

void register_runtime(pybind11::module& m) {
  pybind11::class_<PageAllocator>(m, "PageAllocator")
      .def(pybind11::init<int64_t, int64_t>())
      .def("num_free", &PageAllocator::num_free)
      .def("num_pages", &PageAllocator::num_pages)
      .def("page_size", &PageAllocator::page_size)
      .def("ensure", &PageAllocator::ensure)
      .def("fork_prefix", &PageAllocator::fork_prefix)
      .def("release", &PageAllocator::release)
      .def("pages", &PageAllocator::pages)
      .def("fill_row", &PageAllocator::fill_row);
}
