// Native paged-KV bookkeeping for the drafter route pool and the target sequence.
//
// Design (B200 build, not a port of the reference's SGLang bridge):
//  * PagePool: a fixed set of KV pages shared by every layer (a page id indexes
//    the same page in each layer's cache), a free stack, a per-page reference
//    count and a per-page high-water mark (number of leading slots that hold
//    data written by some view).
//  * RoutePool: one committed prefix (a page list, the last page possibly
//    partial) plus live routes.  A route shares the prefix's full pages
//    implicitly and owns a short list of "tail" pages covering positions from
//    the prefix's first non-full page onward.  Forking copies that short list;
//    it never touches the prefix's O(P/page) pages.
//  * Writer lease: a view may append in place into a partial page if it holds
//    the only reference or if its valid length in the page equals the page's
//    high-water mark and nobody claimed that slot before it in the same batch.
//    Every other writer gets a private page with the valid tail copied first
//    (tail-page copy-on-write).  N writers of one partial page therefore cause
//    N-1 copies; full pages are never copied.
//  * Reclamation is eager (reference counts); prune() is a mark-and-sweep
//    safety net used by validators and tests.
//
// Behavioural parity: reference src/atlas_0709/flashinfer_paged/sglang_runtime.py
// lines 89-1117 (prepare_frontier, tail COW at 708-798, commit_route_as_prefix at
// 357-378, release_unreferenced_node_slots at 507-539, page_reference_counts at
// 380-396, validate_route_physical_state at 398-477).

#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace {

class PagePool {
 public:
  PagePool(int64_t num_pages, int64_t page_size) : page_size_(page_size) {
    if (num_pages <= 0 || page_size <= 0) throw std::invalid_argument("num_pages and page_size must be positive");
    refcnt_.assign(num_pages, 0);
    hw_.assign(num_pages, 0);
    free_.reserve(num_pages);
    for (int64_t p = num_pages - 1; p >= 0; --p) free_.push_back(static_cast<int32_t>(p));
  }

  int32_t alloc() {
    if (free_.empty()) throw std::runtime_error("KV page pool exhausted");
    int32_t p = free_.back();
    free_.pop_back();
    refcnt_[p] = 1;
    hw_[p] = 0;
    ++allocs_;
    return p;
  }
  void incref(int32_t p) {
    check(p);
    if (refcnt_[p] <= 0) throw std::runtime_error("incref of a free page");
    ++refcnt_[p];
  }
  // Returns true when the page went back to the free stack.
  bool decref(int32_t p) {
    check(p);
    if (refcnt_[p] <= 0) throw std::runtime_error("decref of a free page");
    if (--refcnt_[p] == 0) {
      free_.push_back(p);
      ++frees_;
      return true;
    }
    return false;
  }
  int32_t refcount(int32_t p) const {
    check(p);
    return refcnt_[p];
  }
  int32_t& hw(int32_t p) {
    check(p);
    return hw_[p];
  }
  int64_t num_pages() const { return static_cast<int64_t>(refcnt_.size()); }
  int64_t free_pages() const { return static_cast<int64_t>(free_.size()); }
  int64_t used_pages() const { return num_pages() - free_pages(); }
  int64_t page_size() const { return page_size_; }
  int64_t allocs() const { return allocs_; }
  int64_t frees() const { return frees_; }
  // Forcibly return a page (used by mark-and-sweep for leaked pages).
  void force_free(int32_t p) {
    check(p);
    if (refcnt_[p] > 0) {
      refcnt_[p] = 0;
      free_.push_back(p);
      ++frees_;
    }
  }

 private:
  void check(int32_t p) const {
    if (p < 0 || p >= static_cast<int32_t>(refcnt_.size())) throw std::out_of_range("page id out of range");
  }
  int64_t page_size_;
  std::vector<int32_t> refcnt_, hw_, free_;
  int64_t allocs_ = 0, frees_ = 0;
};

struct View {
  std::vector<int32_t> tail;  // pages for page indices >= base (base = prefix full pages at fork time)
  int32_t len = 0;
};

class RoutePool {
 public:
  RoutePool(std::shared_ptr<PagePool> pool) : pool_(std::move(pool)), ps_(static_cast<int32_t>(pool_->page_size())) {}

  // ------------------------------------------------------------------ prefix
  int64_t prefix_len() const { return prefix_len_; }
  torch::Tensor prefix_pages() const { return to_tensor(prefix_pages_); }
  int64_t prefix_full_pages() const { return prefix_len_ / ps_; }

  // Extend the committed prefix by n positions (prefill, fallback EXTEND, target AR).
  // Returns slot ids [n] and the copy plan [m,3] (src page, dst page, tokens).
  std::vector<torch::Tensor> append_prefix(int64_t n) {
    std::vector<int32_t> slots;
    std::vector<int32_t> copies;
    slots.reserve(n);
    for (int64_t i = 0; i < n; ++i) {
      int32_t off = prefix_len_ % ps_;
      int32_t slot;
      if (off == 0) {
        int32_t p = pool_->alloc();
        pool_->hw(p) = 1;
        prefix_pages_.push_back(p);
        slot = p * ps_;
      } else {
        int32_t& p = prefix_pages_.back();
        slot = claim_or_copy(p, off, copies);
      }
      slots.push_back(slot);
      ++prefix_len_;
    }
    return {to_tensor(slots), copy_tensor(copies)};
  }

  // Make sure prefix pages back positions [0, total) without changing prefix_len
  // (target scratch region for tree nodes and AR tokens).  Returns slot ids of
  // positions [prefix_len, total).  Only valid when no route shares the tail.
  torch::Tensor reserve_scratch(int64_t total) {
    if (!routes_.empty()) throw std::runtime_error("reserve_scratch requires a route-free pool");
    int64_t need_pages = (total + ps_ - 1) / ps_;
    while (static_cast<int64_t>(prefix_pages_.size()) < need_pages) {
      int32_t p = pool_->alloc();
      prefix_pages_.push_back(p);
    }
    std::vector<int32_t> slots;
    for (int64_t pos = prefix_len_; pos < total; ++pos) slots.push_back(prefix_pages_[pos / ps_] * ps_ + pos % ps_);
    return to_tensor(slots);
  }

  // Set the committed length inside already reserved pages and free pages beyond.
  void set_prefix_len(int64_t n) {
    if (!routes_.empty()) throw std::runtime_error("set_prefix_len requires a route-free pool");
    int64_t cap = static_cast<int64_t>(prefix_pages_.size()) * ps_;
    if (n < 0 || n > cap) throw std::out_of_range("set_prefix_len beyond reserved pages");
    prefix_len_ = n;
    int64_t keep = (n + ps_ - 1) / ps_;
    while (static_cast<int64_t>(prefix_pages_.size()) > keep) {
      pool_->decref(prefix_pages_.back());
      prefix_pages_.pop_back();
    }
    if (!prefix_pages_.empty() && (n % ps_)) pool_->hw(prefix_pages_.back()) = static_cast<int32_t>(n % ps_);
  }

  torch::Tensor slots_for_positions(int64_t start, int64_t count) const {
    std::vector<int32_t> s;
    s.reserve(count);
    for (int64_t pos = start; pos < start + count; ++pos) {
      int64_t pi = pos / ps_;
      if (pi >= static_cast<int64_t>(prefix_pages_.size())) throw std::out_of_range("position beyond prefix pages");
      s.push_back(prefix_pages_[pi] * ps_ + static_cast<int32_t>(pos % ps_));
    }
    return to_tensor(s);
  }

  // ------------------------------------------------------------------ routes
  void fork_from_prefix(int64_t rid) {
    if (routes_.count(rid)) throw std::runtime_error("route already exists");
    View v;
    v.len = static_cast<int32_t>(prefix_len_);
    if (prefix_len_ % ps_) {
      int32_t p = prefix_pages_.back();
      pool_->incref(p);
      v.tail.push_back(p);
    }
    routes_.emplace(rid, std::move(v));
  }

  void fork(int64_t child, int64_t parent) {
    auto it = routes_.find(parent);
    if (it == routes_.end()) throw std::runtime_error("fork from unknown route");
    if (routes_.count(child)) throw std::runtime_error("route already exists");
    View v = it->second;
    for (int32_t p : v.tail) pool_->incref(p);
    routes_.emplace(child, std::move(v));
  }

  bool has_route(int64_t rid) const { return routes_.count(rid) != 0; }
  int64_t route_len(int64_t rid) const { return get(rid).len; }
  torch::Tensor route_tail_pages(int64_t rid) const { return to_tensor(get(rid).tail); }
  int64_t num_routes() const { return static_cast<int64_t>(routes_.size()); }

  int64_t release(int64_t rid) {
    auto it = routes_.find(rid);
    if (it == routes_.end()) return 0;
    int64_t freed = 0;
    for (int32_t p : it->second.tail) freed += pool_->decref(p);
    routes_.erase(it);
    refresh_prefix_lease();
    return freed;
  }

  // Keep only the listed routes.  Returns {released routes, freed pages}.
  std::vector<int64_t> retain(const std::vector<int64_t>& keep) {
    std::unordered_set<int64_t> k(keep.begin(), keep.end());
    std::vector<int64_t> drop;
    for (auto& kv : routes_)
      if (!k.count(kv.first)) drop.push_back(kv.first);
    std::sort(drop.begin(), drop.end());
    int64_t freed = 0;
    for (int64_t r : drop) freed += release(r);
    return {static_cast<int64_t>(drop.size()), freed};
  }

  // Plan one appended token for each route (in batch order).  Returns
  // slot ids [B] and the copy plan [m,3]; route lengths advance by one.
  std::vector<torch::Tensor> prepare_append(const std::vector<int64_t>& rids) {
    std::vector<int32_t> slots;
    std::vector<int32_t> copies;
    slots.reserve(rids.size());
    const int64_t base = prefix_len_ / ps_;
    for (int64_t rid : rids) {
      View& v = get(rid);
      int32_t off = v.len % ps_;
      int64_t idx = v.len / ps_ - base;
      int32_t slot;
      if (off == 0) {
        if (idx != static_cast<int64_t>(v.tail.size())) throw std::runtime_error("route tail pages out of sync");
        int32_t p = pool_->alloc();
        pool_->hw(p) = 1;
        v.tail.push_back(p);
        slot = p * ps_;
      } else {
        if (idx != static_cast<int64_t>(v.tail.size()) - 1) throw std::runtime_error("route tail pages out of sync");
        slot = claim_or_copy(v.tail.back(), off, copies);
      }
      slots.push_back(slot);
      ++v.len;
    }
    return {to_tensor(slots), copy_tensor(copies)};
  }

  // Per-row attention descriptors: tail page table [B, max_tail] (padded with
  // the row's last page) and lengths [B].  Logical page j of row b is
  // prefix_pages[j] for j < prefix_full_pages and tail[b][j - prefix_full_pages] after.
  std::vector<torch::Tensor> row_tables(const std::vector<int64_t>& rids, int64_t max_tail) const {
    const int64_t b = static_cast<int64_t>(rids.size());
    auto tails = torch::zeros({b, max_tail}, torch::dtype(torch::kInt32));
    auto lens = torch::zeros({b}, torch::dtype(torch::kInt32));
    auto* tp = tails.data_ptr<int32_t>();
    auto* lp = lens.data_ptr<int32_t>();
    for (int64_t i = 0; i < b; ++i) {
      const View& v = get(rids[i]);
      if (static_cast<int64_t>(v.tail.size()) > max_tail) throw std::runtime_error("route tail longer than max_tail");
      int32_t last = v.tail.empty() ? 0 : v.tail.back();
      for (int64_t j = 0; j < max_tail; ++j) tp[i * max_tail + j] = j < static_cast<int64_t>(v.tail.size()) ? v.tail[j] : last;
      lp[i] = v.len;
    }
    return {tails, lens};
  }

  // Promote a route's pages to the committed prefix (zero copy) and rebase the
  // other live routes, which must extend the committed route.  The committed
  // route itself is released.  Returns freed pages.
  int64_t commit(int64_t rid) {
    View r = get(rid);
    const int64_t old_base = prefix_len_ / ps_;
    const int64_t new_len = r.len;
    const int64_t new_base = new_len / ps_;
    const int64_t drop = new_base - old_base;
    for (auto& kv : routes_) {
      if (kv.first == rid) continue;
      View& v = kv.second;
      if (v.len < new_len || static_cast<int64_t>(v.tail.size()) < drop)
        throw std::runtime_error("cannot rebase a route that does not extend the committed route");
      for (int64_t i = 0; i < drop; ++i)
        if (v.tail[i] != r.tail[i]) throw std::runtime_error("retained route does not share the committed full pages");
    }
    // New prefix pages: old full pages + the committed route's tail.
    int64_t freed = 0;
    if (prefix_len_ % ps_) {
      freed += pool_->decref(prefix_pages_.back());
      prefix_pages_.pop_back();
    }
    for (int32_t p : r.tail) {
      pool_->incref(p);
      prefix_pages_.push_back(p);
    }
    prefix_len_ = new_len;
    for (auto& kv : routes_) {
      if (kv.first == rid) continue;
      View& v = kv.second;
      for (int64_t i = 0; i < drop; ++i) freed += pool_->decref(v.tail[i]);
      v.tail.erase(v.tail.begin(), v.tail.begin() + drop);
    }
    freed += release(rid);
    return freed;
  }

  // Drop the prefix and every route (session end / reset).
  int64_t clear() {
    int64_t freed = 0;
    std::vector<int64_t> ids;
    for (auto& kv : routes_) ids.push_back(kv.first);
    for (int64_t r : ids) freed += release(r);
    for (int32_t p : prefix_pages_) freed += pool_->decref(p);
    prefix_pages_.clear();
    prefix_len_ = 0;
    return freed;
  }

  // ------------------------------------------------------------- validation
  // Reference counts recomputed from the views: {page: count}.
  std::unordered_map<int32_t, int32_t> recomputed_refcounts() const {
    std::unordered_map<int32_t, int32_t> c;
    for (int32_t p : prefix_pages_) ++c[p];
    for (auto& kv : routes_)
      for (int32_t p : kv.second.tail) ++c[p];
    return c;
  }

  // Checks every route's length/page layout and that stored reference counts
  // cover the recomputed ones.  Throws with a description on violation.
  void validate() const {
    const int64_t base = prefix_len_ / ps_;
    if (static_cast<int64_t>(prefix_pages_.size()) != (prefix_len_ + ps_ - 1) / ps_) {
      std::ostringstream os;
      os << "prefix page count " << prefix_pages_.size() << " does not cover prefix length " << prefix_len_;
      throw std::runtime_error(os.str());
    }
    for (auto& kv : routes_) {
      const View& v = kv.second;
      int64_t need = (v.len + ps_ - 1) / ps_ - base;
      if (v.len < prefix_len_ || static_cast<int64_t>(v.tail.size()) != need) {
        std::ostringstream os;
        os << "route " << kv.first << " physical length does not match logical KV: len=" << v.len
           << " tail_pages=" << v.tail.size() << " expected=" << need;
        throw std::runtime_error(os.str());
      }
    }
    for (auto& pc : recomputed_refcounts()) {
      if (pool_->refcount(pc.first) < pc.second) {
        std::ostringstream os;
        os << "page " << pc.first << " has refcount " << pool_->refcount(pc.first) << " < " << pc.second << " views";
        throw std::runtime_error(os.str());
      }
    }
  }

  std::shared_ptr<PagePool> pool() const { return pool_; }
  int64_t cow_pages_copied() const { return cow_pages_; }
  int64_t cow_tokens_copied() const { return cow_tokens_; }
  int64_t in_place_appends() const { return in_place_; }

 private:
  View& get(int64_t rid) {
    auto it = routes_.find(rid);
    if (it == routes_.end()) throw std::runtime_error("unknown route id");
    return it->second;
  }
  const View& get(int64_t rid) const {
    auto it = routes_.find(rid);
    if (it == routes_.end()) throw std::runtime_error("unknown route id");
    return it->second;
  }

  // Claim slot `off` of partial page `p` (in place) or copy-on-write it.
  int32_t claim_or_copy(int32_t& p, int32_t off, std::vector<int32_t>& copies) {
    if (pool_->refcount(p) == 1) {
      pool_->hw(p) = off + 1;
      ++in_place_;
      return p * ps_ + off;
    }
    if (pool_->hw(p) == off) {
      pool_->hw(p) = off + 1;
      ++in_place_;
      return p * ps_ + off;
    }
    int32_t q = pool_->alloc();
    copies.push_back(p);
    copies.push_back(q);
    copies.push_back(off);
    pool_->decref(p);
    pool_->hw(q) = off + 1;
    p = q;
    ++cow_pages_;
    cow_tokens_ += off;
    return q * ps_ + off;
  }

  // When the prefix is the sole holder of its partial page again, forget any
  // slots written by released routes so the next writer gets the lease.
  void refresh_prefix_lease() {
    if (prefix_len_ % ps_ && !prefix_pages_.empty()) {
      int32_t p = prefix_pages_.back();
      if (pool_->refcount(p) == 1) pool_->hw(p) = static_cast<int32_t>(prefix_len_ % ps_);
    }
  }

  static torch::Tensor to_tensor(const std::vector<int32_t>& v) {
    auto t = torch::empty({static_cast<int64_t>(v.size())}, torch::dtype(torch::kInt32));
    if (!v.empty()) std::copy(v.begin(), v.end(), t.data_ptr<int32_t>());
    return t;
  }
  static torch::Tensor copy_tensor(const std::vector<int32_t>& v) {
    auto t = torch::empty({static_cast<int64_t>(v.size() / 3), 3}, torch::dtype(torch::kInt32));
    if (!v.empty()) std::copy(v.begin(), v.end(), t.data_ptr<int32_t>());
    return t;
  }

  std::shared_ptr<PagePool> pool_;
  int32_t ps_;
  std::vector<int32_t> prefix_pages_;
  int64_t prefix_len_ = 0;
  std::unordered_map<int64_t, View> routes_;
  int64_t cow_pages_ = 0, cow_tokens_ = 0, in_place_ = 0;
};

// ------------------------------------------------------------- tree dedup
// Prefix trie over equal-depth paths: one node per unique token prefix.
// Returns tokens [N], parents [N] (-1 = root), depths [N], route->node paths
// [R, D] and a 64-bit ancestor mask per node (bit j set when node j is an
// ancestor of, or equal to, the node).  Parity: reference
// src/atlas_0709/flashinfer_full_verify.py:570-616 (trie) and :719-724 (mask).
std::vector<torch::Tensor> build_tree(torch::Tensor paths) {
  TORCH_CHECK(paths.dim() == 2 && paths.scalar_type() == torch::kInt64, "paths must be int64 [R, D]");
  auto pc = paths.contiguous();
  const int64_t R = pc.size(0), D = pc.size(1);
  TORCH_CHECK(R > 0 && D > 0, "paths must be non-empty");
  const int64_t* tp = pc.data_ptr<int64_t>();
  std::vector<int64_t> tok;
  std::vector<int32_t> par, dep;
  std::vector<std::unordered_map<int64_t, int32_t>> kids;
  std::unordered_map<int64_t, int32_t> root;
  auto node_paths = torch::empty({R, D}, torch::dtype(torch::kInt32));
  auto* np = node_paths.data_ptr<int32_t>();
  for (int64_t r = 0; r < R; ++r) {
    int32_t parent = -1;
    for (int64_t d = 0; d < D; ++d) {
      int64_t t = tp[r * D + d];
      auto& children = parent < 0 ? root : kids[parent];
      auto it = children.find(t);
      int32_t n;
      if (it == children.end()) {
        n = static_cast<int32_t>(tok.size());
        children.emplace(t, n);
        tok.push_back(t);
        par.push_back(parent);
        dep.push_back(static_cast<int32_t>(d));
        kids.emplace_back();
      } else {
        n = it->second;
      }
      np[r * D + d] = n;
      parent = n;
    }
  }
  const int64_t N = static_cast<int64_t>(tok.size());
  auto tokens = torch::empty({N}, torch::dtype(torch::kInt64));
  auto parents = torch::empty({N}, torch::dtype(torch::kInt32));
  auto depths = torch::empty({N}, torch::dtype(torch::kInt32));
  std::copy(tok.begin(), tok.end(), tokens.data_ptr<int64_t>());
  std::copy(par.begin(), par.end(), parents.data_ptr<int32_t>());
  std::copy(dep.begin(), dep.end(), depths.data_ptr<int32_t>());
  // Ancestor masks as [N, W] uint64 words stored in int64 (W = ceil(N/64)).
  const int64_t W = (N + 63) / 64;
  auto masks = torch::zeros({N, W}, torch::dtype(torch::kInt64));
  auto* mp = reinterpret_cast<uint64_t*>(masks.data_ptr<int64_t>());
  for (int64_t i = 0; i < N; ++i) {
    for (int32_t a = static_cast<int32_t>(i); a >= 0; a = par[a]) mp[i * W + a / 64] |= (uint64_t(1) << (a % 64));
  }
  return {tokens, parents, depths, node_paths, masks};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "Native paged-KV bookkeeping (page pool, route views, tail COW lease, tree dedup)";
  pybind11::class_<PagePool, std::shared_ptr<PagePool>>(m, "PagePool")
      .def(pybind11::init<int64_t, int64_t>(), pybind11::arg("num_pages"), pybind11::arg("page_size"))
      .def("alloc", &PagePool::alloc)
      .def("incref", &PagePool::incref)
      .def("decref", &PagePool::decref)
      .def("refcount", &PagePool::refcount)
      .def("high_water", [](PagePool& p, int32_t page) { return p.hw(page); })
      .def("force_free", &PagePool::force_free)
      .def_property_readonly("num_pages", &PagePool::num_pages)
      .def_property_readonly("free_pages", &PagePool::free_pages)
      .def_property_readonly("used_pages", &PagePool::used_pages)
      .def_property_readonly("page_size", &PagePool::page_size)
      .def_property_readonly("allocs", &PagePool::allocs)
      .def_property_readonly("frees", &PagePool::frees);
  pybind11::class_<RoutePool>(m, "RoutePool")
      .def(pybind11::init<std::shared_ptr<PagePool>>())
      .def_property_readonly("prefix_len", &RoutePool::prefix_len)
      .def_property_readonly("prefix_full_pages", &RoutePool::prefix_full_pages)
      .def("prefix_pages", &RoutePool::prefix_pages)
      .def("append_prefix", &RoutePool::append_prefix)
      .def("reserve_scratch", &RoutePool::reserve_scratch)
      .def("set_prefix_len", &RoutePool::set_prefix_len)
      .def("slots_for_positions", &RoutePool::slots_for_positions)
      .def("fork_from_prefix", &RoutePool::fork_from_prefix)
      .def("fork", &RoutePool::fork)
      .def("has_route", &RoutePool::has_route)
      .def("route_len", &RoutePool::route_len)
      .def("route_tail_pages", &RoutePool::route_tail_pages)
      .def_property_readonly("num_routes", &RoutePool::num_routes)
      .def("release", &RoutePool::release)
      .def("retain", &RoutePool::retain)
      .def("prepare_append", &RoutePool::prepare_append)
      .def("row_tables", &RoutePool::row_tables)
      .def("commit", &RoutePool::commit)
      .def("clear", &RoutePool::clear)
      .def("recomputed_refcounts", &RoutePool::recomputed_refcounts)
      .def("validate", &RoutePool::validate)
      .def_property_readonly("pool", &RoutePool::pool)
      .def_property_readonly("cow_pages_copied", &RoutePool::cow_pages_copied)
      .def_property_readonly("cow_tokens_copied", &RoutePool::cow_tokens_copied)
      .def_property_readonly("in_place_appends", &RoutePool::in_place_appends);
  m.def("build_tree", &build_tree, "Deduplicate equal-depth paths into a trie with ancestor masks");
}
