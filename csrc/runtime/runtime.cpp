// Host-side runtime pieces of the serving engine (module sglang_omni_b200._runtime):
//
//  * PageAllocator  - free-list allocator of KV-cache pages with per-owner
//                     accounting (the paged KV pool of every AR stage);
//  * DecodeMetaBuilder - fills the packed int32 metadata of one decode step
//                     (kv lengths, slot mapping, M-RoPE positions, block table
//                     rows, request slots) into a caller-provided pinned buffer,
//                     allocating a page whenever a request crosses a page edge;
//  * ShmRing        - single-producer / single-consumer byte ring in POSIX
//                     shared memory used by the CPU relay between stage processes.
//
// Reference counterparts: SGLang's token-to-KV pool and ScheduleBatch metadata
// (used through sglang_omni/engines/ar/sglang_backend/scheduler/*.py) and the
// POSIX SHM relay (sglang_omni/relay/shm.py:18-169).
#include <fcntl.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

class PageAllocator {
 public:
  explicit PageAllocator(int num_pages, int reserved) : num_pages_(num_pages) {
    if (reserved < 0 || reserved > num_pages) throw std::invalid_argument("bad reserved page count");
    free_.reserve(num_pages);
    for (int p = num_pages - 1; p >= reserved; --p) free_.push_back(p);
  }
  int num_free() const { return static_cast<int>(free_.size()); }
  int num_pages() const { return num_pages_; }
  bool can_alloc(int n) const { return n <= static_cast<int>(free_.size()); }
  std::vector<int> alloc(int n) {
    if (n > static_cast<int>(free_.size())) throw std::runtime_error("KV pool out of pages");
    std::vector<int> out(free_.end() - n, free_.end());
    free_.resize(free_.size() - n);
    return out;
  }
  int alloc_one() {
    if (free_.empty()) return -1;
    int p = free_.back();
    free_.pop_back();
    return p;
  }
  void free(const std::vector<int>& pages) {
    for (int p : pages) {
      if (p < 0 || p >= num_pages_) throw std::out_of_range("page id out of range");
      free_.push_back(p);
    }
  }

 private:
  int num_pages_;
  std::vector<int> free_;
};

// Packed layout (int32), for a batch of B rows and P pages per row:
//   [0, B)            kv_lens (after this step's token)
//   [B, 2B)           slot_mapping
//   [2B, 5B)          positions rows t, h, w
//   [5B, 6B)          request slot ids
//   [6B, 6B + B*P)    block table rows
class DecodeMetaBuilder {
 public:
  DecodeMetaBuilder(int max_batch, int max_pages) : max_batch_(max_batch), max_pages_(max_pages) {}
  static int packed_size(int batch, int pages) { return 6 * batch + batch * pages; }

  // kv_len_before[i]: tokens already in the cache; pages[i]: page list (appended
  // in place when a new page is needed); returns the number of rows written.
  int build(py::array_t<int32_t, py::array::c_style> out, py::list pages, py::array_t<int64_t> kv_len_before,
            py::array_t<int64_t> mrope_delta, py::array_t<int64_t> slots, PageAllocator& alloc, int padded_batch) {
    auto o = out.mutable_unchecked<1>();
    auto kl = kv_len_before.unchecked<1>();
    auto md = mrope_delta.unchecked<1>();
    auto sl = slots.unchecked<1>();
    const int B = static_cast<int>(kl.shape(0));
    if (padded_batch < B || padded_batch > max_batch_) throw std::invalid_argument("bad padded batch");
    const int PB = padded_batch, P = max_pages_;
    if (o.shape(0) < packed_size(PB, P)) throw std::invalid_argument("packed buffer too small");
    for (int i = 0; i < B; ++i) {
      py::list pl = pages[i];
      const int64_t pos = kl(i);
      const int page_idx = static_cast<int>(pos / 64);
      if (page_idx >= P) throw std::runtime_error("request exceeds max pages");
      if (page_idx >= static_cast<int>(pl.size())) {
        const int p = alloc.alloc_one();
        if (p < 0) throw std::runtime_error("KV pool out of pages");
        pl.append(p);
      }
      const int page = pl[page_idx].cast<int>();
      o(i) = static_cast<int32_t>(pos + 1);
      o(PB + i) = page * 64 + static_cast<int>(pos % 64);
      const int32_t p3 = static_cast<int32_t>(pos + md(i));
      o(2 * PB + i) = p3;
      o(3 * PB + i) = p3;
      o(4 * PB + i) = p3;
      o(5 * PB + i) = static_cast<int32_t>(sl(i));
      int32_t* row = &o(6 * PB + i * P);
      const int n = static_cast<int>(pl.size());
      for (int j = 0; j < n && j < P; ++j) row[j] = pl[j].cast<int32_t>();
      for (int j = n; j < P; ++j) row[j] = 0;
    }
    for (int i = B; i < PB; ++i) {  // padding rows: empty context, no cache write, dummy slot 0
      o(i) = 0;
      o(PB + i) = -1;
      o(2 * PB + i) = o(3 * PB + i) = o(4 * PB + i) = 0;
      o(5 * PB + i) = 0;
      std::memset(&o(6 * PB + i * P), 0, sizeof(int32_t) * P);
    }
    return B;
  }

 private:
  int max_batch_, max_pages_;
};

// SPSC byte ring in POSIX shared memory: [head u64][tail u64][capacity bytes].
class ShmRing {
 public:
  ShmRing(const std::string& name, size_t capacity, bool create) : name_(name), cap_(capacity), owner_(create) {
    const int flags = create ? (O_CREAT | O_RDWR) : O_RDWR;
    fd_ = shm_open(name.c_str(), flags, 0600);
    if (fd_ < 0) throw std::runtime_error("shm_open failed: " + name);
    const size_t total = 64 + capacity;
    if (create && ftruncate(fd_, static_cast<off_t>(total)) != 0) throw std::runtime_error("ftruncate failed");
    base_ = static_cast<uint8_t*>(mmap(nullptr, total, PROT_READ | PROT_WRITE, MAP_SHARED, fd_, 0));
    if (base_ == MAP_FAILED) throw std::runtime_error("mmap failed");
    if (create) {
      head()->store(0);
      tail()->store(0);
    }
  }
  ~ShmRing() {
    if (base_ && base_ != MAP_FAILED) munmap(base_, 64 + cap_);
    if (fd_ >= 0) close(fd_);
    if (owner_) shm_unlink(name_.c_str());
  }
  size_t capacity() const { return cap_; }
  size_t readable() const { return tail()->load(std::memory_order_acquire) - head()->load(std::memory_order_acquire); }
  // Writes one length-prefixed message; returns false when there is no room.
  bool put(py::bytes data) {
    std::string s = data;
    const uint64_t need = 8 + s.size();
    const uint64_t t = tail()->load(std::memory_order_relaxed);
    const uint64_t h = head()->load(std::memory_order_acquire);
    if (need > cap_ - (t - h)) return false;
    uint64_t len = s.size();
    copy_in(t, reinterpret_cast<const uint8_t*>(&len), 8);
    copy_in(t + 8, reinterpret_cast<const uint8_t*>(s.data()), s.size());
    tail()->store(t + need, std::memory_order_release);
    return true;
  }
  py::object get() {
    const uint64_t h = head()->load(std::memory_order_relaxed);
    const uint64_t t = tail()->load(std::memory_order_acquire);
    if (t - h < 8) return py::none();
    uint64_t len = 0;
    copy_out(h, reinterpret_cast<uint8_t*>(&len), 8);
    std::string s(len, '\0');
    copy_out(h + 8, reinterpret_cast<uint8_t*>(&s[0]), len);
    head()->store(h + 8 + len, std::memory_order_release);
    return py::bytes(s);
  }

 private:
  std::atomic<uint64_t>* head() const { return reinterpret_cast<std::atomic<uint64_t>*>(base_); }
  std::atomic<uint64_t>* tail() const { return reinterpret_cast<std::atomic<uint64_t>*>(base_ + 8); }
  void copy_in(uint64_t pos, const uint8_t* src, size_t n) {
    uint8_t* data = base_ + 64;
    for (size_t done = 0; done < n;) {
      const size_t off = (pos + done) % cap_;
      const size_t chunk = std::min(n - done, cap_ - off);
      std::memcpy(data + off, src + done, chunk);
      done += chunk;
    }
  }
  void copy_out(uint64_t pos, uint8_t* dst, size_t n) const {
    const uint8_t* data = base_ + 64;
    for (size_t done = 0; done < n;) {
      const size_t off = (pos + done) % cap_;
      const size_t chunk = std::min(n - done, cap_ - off);
      std::memcpy(dst + done, data + off, chunk);
      done += chunk;
    }
  }
  std::string name_;
  size_t cap_;
  bool owner_;
  int fd_ = -1;
  uint8_t* base_ = nullptr;
};

PYBIND11_MODULE(_runtime, m) {
  m.doc() = "host runtime of sglang_omni_b200 (page allocator, decode metadata, shm ring)";
  py::class_<PageAllocator>(m, "PageAllocator")
      .def(py::init<int, int>(), py::arg("num_pages"), py::arg("reserved") = 1)
      .def("num_free", &PageAllocator::num_free)
      .def("num_pages", &PageAllocator::num_pages)
      .def("can_alloc", &PageAllocator::can_alloc)
      .def("alloc", &PageAllocator::alloc)
      .def("alloc_one", &PageAllocator::alloc_one)
      .def("free", &PageAllocator::free);
  py::class_<DecodeMetaBuilder>(m, "DecodeMetaBuilder")
      .def(py::init<int, int>())
      .def_static("packed_size", &DecodeMetaBuilder::packed_size)
      .def("build", &DecodeMetaBuilder::build);
  py::class_<ShmRing>(m, "ShmRing")
      .def(py::init<const std::string&, size_t, bool>(), py::arg("name"), py::arg("capacity"), py::arg("create"))
      .def("capacity", &ShmRing::capacity)
      .def("readable", &ShmRing::readable)
      .def("put", &ShmRing::put)
      .def("get", &ShmRing::get);
}
