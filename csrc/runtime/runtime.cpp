// Host-side runtime pieces of the serving engine (module sglang_omni_b200._runtime):
//
//  * PageAllocator  - free-list allocator of KV-cache pages with per-owner
//                     accounting (the paged KV pool of every AR stage);
//  * DecodeMetaBuilder - fills the packed int32 metadata of one decode step
//                     (kv lengths, slot mapping, M-RoPE positions, block table
//                     rows, request slots) into a caller-provided pinned buffer,
//                     allocating a page whenever a request crosses a page edge;
//  * ShmRing        - single-producer / single-consumer byte ring in POSIX
//                     shared memory used by the CPU relay between stage processes;
//  * PrefixCache    - page-granular radix tree of cached KV prefixes: each node is
//                     one full 64-token page, shared by every request whose prompt
//                     starts with the same token blocks (same namespace), locked
//                     while a request uses it and evicted leaf-first in LRU order
//                     when the page allocator runs dry.
//
// Reference counterparts: SGLang's token-to-KV pool and ScheduleBatch metadata
// (used through sglang_omni/engines/ar/sglang_backend/scheduler/*.py) and the
// POSIX SHM relay (sglang_omni/relay/shm.py:18-169); SGLang's RadixCache as the
// engines create it (sglang_omni/engines/ar/sglang_backend/scheduler/cache.py:9-30,
// cache_unfinished_req at sglang_omni/engines/omni/runtime/sglang_ar.py:205).
#include <fcntl.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <queue>
#include <unordered_map>
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

// Radix tree over page-sized token blocks.  The key of a node is
// (parent node, namespace, the block's token ids); a lookup hashes the key and
// compares the stored ids, so hash collisions never alias two prefixes.
// A request that matched a prefix holds one reference on every node of its
// path (ancestors of a referenced node are therefore always referenced), and
// a node is evictable once it has no reference and no child.
class PrefixCache {
 public:
  explicit PrefixCache(int block) : block_(block) {
    if (block <= 0) throw std::invalid_argument("block must be positive");
    nodes_.push_back(Node{});  // node 0: root (never evicted, holds no page)
  }

  int block() const { return block_; }
  int cached_pages() const { return live_; }
  int evictable_pages() const {
    int n = 0;
    for (size_t i = 1; i < nodes_.size(); ++i)
      if (nodes_[i].alive && nodes_[i].ref == 0) ++n;
    return n;
  }
  uint64_t hits() const { return hit_blocks_; }

  // Longest cached run of full blocks at the start of `tokens` (at most
  // max_blocks blocks).  Takes a reference on every matched node and returns
  // (node ids, page ids) in order.
  py::tuple match(uint64_t ns, py::array_t<int32_t, py::array::c_style> tokens, int max_blocks) {
    auto t = tokens.unchecked<1>();
    const int nblk = std::min<int>(max_blocks, static_cast<int>(t.shape(0)) / block_);
    std::vector<int> path, pages;
    int cur = 0;
    const uint64_t now = ++clock_;
    for (int b = 0; b < nblk; ++b) {
      const int32_t* blk = t.data(b * block_);
      const int child = find(cur, ns, blk);
      if (child < 0) break;
      path.push_back(child);
      pages.push_back(nodes_[child].page);
      cur = child;
    }
    for (int n : path) {
      nodes_[n].ref += 1;
      nodes_[n].last = now;
    }
    hit_blocks_ += path.size();
    return py::make_tuple(path, pages);
  }

  // Inserts the full blocks of `tokens` whose KV lives in `pages` (the request's
  // page list, block i in pages[i]); the first locked.size() blocks are the
  // nodes the request matched.  Releases the request's references and returns
  // the pages the caller must free: pages of blocks that another request has
  // cached in the meantime.  Pages that became tree nodes are owned by the cache.
  std::vector<int> insert_release(uint64_t ns, py::array_t<int32_t, py::array::c_style> tokens,
                                  const std::vector<int>& pages, const std::vector<int>& locked) {
    auto t = tokens.unchecked<1>();
    const int nblk = std::min<int>(static_cast<int>(t.shape(0)) / block_, static_cast<int>(pages.size()));
    if (static_cast<int>(locked.size()) > nblk) throw std::invalid_argument("more locked nodes than blocks");
    std::vector<int> dup;
    const uint64_t now = ++clock_;
    int cur = 0;
    for (int b = 0; b < nblk; ++b) {
      if (b < static_cast<int>(locked.size())) {
        cur = locked[b];
        check_node(cur);
        if (nodes_[cur].page != pages[b]) throw std::invalid_argument("locked node does not own the request's page");
        continue;
      }
      const int32_t* blk = t.data(b * block_);
      const int child = find(cur, ns, blk);
      if (child >= 0) {  // cached by another request: keep the tree's copy
        dup.push_back(pages[b]);
        nodes_[child].last = now;
        cur = child;
        continue;
      }
      cur = add(cur, ns, blk, pages[b], now);
    }
    release(locked);
    return dup;
  }

  // Drops the request's references without inserting anything.
  void release(const std::vector<int>& locked) {
    for (int n : locked) {
      check_node(n);
      if (nodes_[n].ref <= 0) throw std::runtime_error("prefix node released more often than matched");
      nodes_[n].ref -= 1;
    }
  }

  // Evicts up to n unreferenced leaves, least recently used first (a parent
  // that becomes an unreferenced leaf joins the queue); returns their pages.
  std::vector<int> evict(int n) {
    using Item = std::pair<uint64_t, int>;
    std::priority_queue<Item, std::vector<Item>, std::greater<Item>> q;
    for (size_t i = 1; i < nodes_.size(); ++i) {
      const Node& x = nodes_[i];
      if (x.alive && x.ref == 0 && x.children == 0) q.push({x.last, static_cast<int>(i)});
    }
    std::vector<int> out;
    while (static_cast<int>(out.size()) < n && !q.empty()) {
      const int id = q.top().second;
      q.pop();
      Node& x = nodes_[id];
      if (!x.alive || x.ref != 0 || x.children != 0) continue;
      out.push_back(x.page);
      const int parent = x.parent;
      remove(id);
      if (parent > 0) {
        const Node& p = nodes_[parent];
        if (p.alive && p.ref == 0 && p.children == 0) q.push({p.last, parent});
      }
    }
    return out;
  }

  // Evicts every unreferenced node; returns their pages.
  std::vector<int> clear() { return evict(static_cast<int>(nodes_.size())); }

 private:
  struct Node {
    int parent = -1;
    int page = -1;
    int ref = 0;
    int children = 0;
    uint64_t ns = 0;
    uint64_t key = 0;
    uint64_t last = 0;
    bool alive = true;
    std::vector<int32_t> toks;
  };

  uint64_t key_of(int parent, uint64_t ns, const int32_t* blk) const {
    // FNV-1a over the parent id, the namespace and the block's token ids.
    uint64_t h = 1469598103934665603ull;
    auto mix = [&h](uint64_t v) {
      for (int i = 0; i < 8; ++i) {
        h ^= (v >> (8 * i)) & 0xffu;
        h *= 1099511628211ull;
      }
    };
    mix(static_cast<uint64_t>(parent));
    mix(ns);
    for (int i = 0; i < block_; ++i) mix(static_cast<uint32_t>(blk[i]));
    return h;
  }

  int find(int parent, uint64_t ns, const int32_t* blk) const {
    auto it = index_.find(key_of(parent, ns, blk));
    if (it == index_.end()) return -1;
    for (int id : it->second) {
      const Node& x = nodes_[id];
      if (x.alive && x.parent == parent && x.ns == ns &&
          std::equal(x.toks.begin(), x.toks.end(), blk))
        return id;
    }
    return -1;
  }

  int add(int parent, uint64_t ns, const int32_t* blk, int page, uint64_t now) {
    int id;
    if (!free_ids_.empty()) {
      id = free_ids_.back();
      free_ids_.pop_back();
    } else {
      id = static_cast<int>(nodes_.size());
      nodes_.push_back(Node{});
    }
    Node& x = nodes_[id];
    x = Node{};
    x.parent = parent;
    x.page = page;
    x.ns = ns;
    x.key = key_of(parent, ns, blk);
    x.last = now;
    x.toks.assign(blk, blk + block_);
    index_[x.key].push_back(id);
    nodes_[parent].children += 1;
    live_ += 1;
    return id;
  }

  void remove(int id) {
    Node& x = nodes_[id];
    auto it = index_.find(x.key);
    if (it != index_.end()) {
      auto& v = it->second;
      v.erase(std::remove(v.begin(), v.end(), id), v.end());
      if (v.empty()) index_.erase(it);
    }
    nodes_[x.parent].children -= 1;
    x.alive = false;
    x.toks.clear();
    x.toks.shrink_to_fit();
    free_ids_.push_back(id);
    live_ -= 1;
  }

  void check_node(int id) const {
    if (id <= 0 || id >= static_cast<int>(nodes_.size()) || !nodes_[id].alive)
      throw std::out_of_range("bad prefix node id");
  }

  int block_;
  int live_ = 0;
  uint64_t clock_ = 0;
  uint64_t hit_blocks_ = 0;
  std::vector<Node> nodes_;
  std::vector<int> free_ids_;
  std::unordered_map<uint64_t, std::vector<int>> index_;
};

PYBIND11_MODULE(_runtime, m) {
  m.doc() = "host runtime of sglang_omni_b200 (page allocator, decode metadata, shm ring, prefix cache)";
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
  py::class_<PrefixCache>(m, "PrefixCache")
      .def(py::init<int>(), py::arg("block") = 64)
      .def("block", &PrefixCache::block)
      .def("cached_pages", &PrefixCache::cached_pages)
      .def("evictable_pages", &PrefixCache::evictable_pages)
      .def("hits", &PrefixCache::hits)
      .def("match", &PrefixCache::match, py::arg("ns"), py::arg("tokens"), py::arg("max_blocks"))
      .def("insert_release", &PrefixCache::insert_release, py::arg("ns"), py::arg("tokens"), py::arg("pages"),
           py::arg("locked"))
      .def("release", &PrefixCache::release)
      .def("evict", &PrefixCache::evict)
      .def("clear", &PrefixCache::clear);
}
