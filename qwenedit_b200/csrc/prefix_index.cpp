// Prefix index for the paged K/V pools: a radix tree over int64 virtual ids, the slot allocator and
// LRU eviction, in one host object.
//
// Behaviour follows what QwenEdit's PagedKVPool (multi_turn/cache/paged.py:52-131) gets from SGLang's
// RadixCache (create_simulated, page_size 1) and TokenToKVPoolAllocator (need_sort=True):
//  * match_prefix walks children keyed by the first token (first page in page mode), splits a node on a
//    partial match and touches every node on the path with one access time (paged.py:75).
//  * insert walks the same way, splitting where the new key diverges, adds one leaf for the new tail and
//    reports how many tokens were already present (paged.py:99-100).
//  * evict collects the leaves depth first, heapifies them on last-access time and pops unlocked leaves
//    until enough tokens are freed, pushing a parent when its last child goes (paged.py:93).
//  * lock refs walk to the root and move tokens between the evictable and protected totals
//    (paged.py:79, :36).
//  * the allocator hands out the head of a sorted free list; freed slots wait in a release list and are
//    merged and sorted only when an allocation needs them (paged.py:91-95, :102).
// Time is a logical clock: every point where the reference reads time.monotonic() (the start of a walk,
// the construction of a node) takes the next tick, so orderings match a clock of unbounded resolution.
//
// Page mode (page_size P > 1, the layout the B200 gather reads through block tables) keeps the same
// structure with keys compared and split in whole pages, keys truncated to whole pages, and the
// allocator handing out whole pages (slot = page * P + offset).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <queue>
#include <vector>

#include "qe_common.h"

namespace qe {

std::string &last_error() {
  static thread_local std::string msg;
  return msg;
}

int fail(int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error() = buf;
  return status;
}

namespace {

struct Node {
  int32_t parent = -1;
  std::vector<int32_t> children;  // insertion order, replaced in place on a split (dict semantics)
  std::vector<int64_t> key;
  std::vector<int64_t> value;
  int64_t lock_ref = 0;
  uint64_t last_access = 0;
  uint32_t gen = 1;
  bool live = false;
};

}  // namespace

struct Index {
  int64_t capacity = 0;  // tokens (page mode: pages * page_size)
  int32_t page = 1;
  int64_t num_pages = 0;  // allocation units (tokens when page == 1)

  std::vector<Node> nodes;
  std::vector<int32_t> free_nodes;
  int32_t root = -1;
  uint64_t clock = 0;
  int64_t evictable = 0;
  int64_t protected_ = 0;
  int64_t live_nodes = 0;

  // allocator state, in allocation units (slots or pages)
  std::vector<int64_t> free_units;  // sorted ascending from free_head on
  size_t free_head = 0;
  std::vector<int64_t> release_units;
  std::vector<uint8_t> unit_free;  // 1 when the unit is in free_units or release_units

  uint64_t tick() { return ++clock; }

  uint64_t handle(int32_t id) const { return (uint64_t(nodes[id].gen) << 32) | uint64_t(uint32_t(id) + 1); }

  int32_t resolve(uint64_t h) const {
    if (h == 0) return -1;
    uint32_t id1 = uint32_t(h & 0xffffffffu);
    uint32_t gen = uint32_t(h >> 32);
    if (id1 == 0 || id1 > nodes.size()) return -1;
    int32_t id = int32_t(id1 - 1);
    const Node &n = nodes[id];
    if (!n.live || n.gen != gen) return -1;
    return id;
  }

  int32_t new_node() {
    int32_t id;
    if (!free_nodes.empty()) {
      id = free_nodes.back();
      free_nodes.pop_back();
    } else {
      id = int32_t(nodes.size());
      nodes.emplace_back();
    }
    Node &n = nodes[id];
    n.parent = -1;
    n.children.clear();
    n.key.clear();
    n.value.clear();
    n.lock_ref = 0;
    n.last_access = tick();  // TreeNode() reads the clock at construction
    n.live = true;
    ++live_nodes;
    return id;
  }

  void drop_node(int32_t id) {
    Node &n = nodes[id];
    n.live = false;
    n.gen += 1;
    if (n.gen == 0) n.gen = 1;
    n.children.clear();
    n.children.shrink_to_fit();
    n.key.clear();
    n.key.shrink_to_fit();
    n.value.clear();
    n.value.shrink_to_fit();
    free_nodes.push_back(id);
    --live_nodes;
  }

  void reset_tree() {
    nodes.clear();
    free_nodes.clear();
    live_nodes = 0;
    root = new_node();
    nodes[root].lock_ref = 1;
    live_nodes = 0;  // the root is not counted
    evictable = 0;
    protected_ = 0;
  }

  void reset_alloc() {
    free_units.resize(size_t(num_pages));
    for (int64_t i = 0; i < num_pages; ++i) free_units[size_t(i)] = i + 1;
    free_head = 0;
    release_units.clear();
    unit_free.assign(size_t(num_pages + 1), 1);
    unit_free[0] = 0;
  }

  // ---- keys ------------------------------------------------------------------------------
  // Child lookup: children are keyed by their first token (page mode: first page).
  int32_t find_child(int32_t node, const int64_t *key) const {
    for (int32_t c : nodes[node].children) {
      const std::vector<int64_t> &ck = nodes[c].key;
      if (page == 1) {
        if (ck[0] == key[0]) return c;
      } else if (std::memcmp(ck.data(), key, sizeof(int64_t) * size_t(page)) == 0) {
        return c;
      }
    }
    return -1;
  }

  // Matched prefix length of node key vs key[0..n) (whole pages in page mode).
  int64_t key_match(const std::vector<int64_t> &a, const int64_t *b, int64_t n) const {
    int64_t m = std::min<int64_t>(int64_t(a.size()), n);
    if (page == 1) {
      int64_t i = 0;
      while (i < m && a[size_t(i)] == b[i]) ++i;
      return i;
    }
    int64_t i = 0;
    while (i + page <= m && std::memcmp(a.data() + i, b + i, sizeof(int64_t) * size_t(page)) == 0) i += page;
    return i;
  }

  // _split_node: the upper `len` tokens of `child` move into a new node between child and its parent.
  int32_t split(int32_t child, int64_t len) {
    int32_t nn = new_node();
    Node &c = nodes[child];
    Node &n = nodes[nn];
    int32_t parent = c.parent;
    n.parent = parent;
    n.lock_ref = c.lock_ref;
    n.key.assign(c.key.begin(), c.key.begin() + len);
    n.value.assign(c.value.begin(), c.value.begin() + len);
    c.key.erase(c.key.begin(), c.key.begin() + len);
    c.value.erase(c.value.begin(), c.value.begin() + len);
    c.parent = nn;
    n.children.push_back(child);
    for (int32_t &slot : nodes[parent].children) {
      if (slot == child) {
        slot = nn;
        break;
      }
    }
    return nn;
  }

  // ---- tree operations -----------------------------------------------------------------------
  int64_t aligned(int64_t n) const { return page == 1 ? n : n / page * page; }

  void match(const int64_t *key, int64_t n, int64_t *out_len, int64_t *out_slots, uint64_t *out_node) {
    n = aligned(n);
    *out_len = 0;
    *out_node = 0;
    if (n <= 0) return;
    uint64_t access = tick();
    int32_t node = root;
    nodes[node].last_access = access;
    int64_t pos = 0, len = 0;
    while (pos < n) {
      int32_t child = find_child(node, key + pos);
      if (child < 0) break;
      nodes[child].last_access = access;
      int64_t plen = key_match(nodes[child].key, key + pos, n - pos);
      if (plen < int64_t(nodes[child].key.size())) {
        int32_t nn = split(child, plen);
        const std::vector<int64_t> &v = nodes[nn].value;
        std::memcpy(out_slots + len, v.data(), v.size() * sizeof(int64_t));
        len += int64_t(v.size());
        node = nn;
        break;
      }
      const std::vector<int64_t> &v = nodes[child].value;
      std::memcpy(out_slots + len, v.data(), v.size() * sizeof(int64_t));
      len += int64_t(v.size());
      node = child;
      pos += plen;
    }
    *out_len = len;
    *out_node = len ? handle(node) : 0;
  }

  int64_t insert(const int64_t *key, const int64_t *value, int64_t n) {
    n = aligned(n);
    uint64_t access = tick();
    int32_t node = root;
    nodes[node].last_access = access;
    if (n <= 0) return 0;
    int64_t pos = 0, total = 0;
    while (pos < n) {
      int32_t child = find_child(node, key + pos);
      if (child < 0) break;
      node = child;
      nodes[node].last_access = access;
      int64_t plen = key_match(nodes[node].key, key + pos, n - pos);
      total += plen;
      pos += plen;
      if (plen < int64_t(nodes[node].key.size())) node = split(node, plen);
    }
    if (pos < n) {
      int32_t leaf = new_node();
      Node &l = nodes[leaf];
      l.parent = node;
      l.key.assign(key + pos, key + n);
      l.value.assign(value + pos, value + n);
      nodes[node].children.push_back(leaf);
      evictable += n - pos;
    }
    return total;
  }

  void lock(int32_t node) {
    while (node != root) {
      Node &x = nodes[node];
      if (x.lock_ref == 0) {
        evictable -= int64_t(x.key.size());
        protected_ += int64_t(x.key.size());
      }
      x.lock_ref += 1;
      node = x.parent;
    }
  }

  bool unlock(int32_t node) {
    for (int32_t v = node; v != root; v = nodes[v].parent)
      if (nodes[v].lock_ref <= 0) return false;
    while (node != root) {
      Node &x = nodes[node];
      if (x.lock_ref == 1) {
        evictable += int64_t(x.key.size());
        protected_ -= int64_t(x.key.size());
      }
      x.lock_ref -= 1;
      node = x.parent;
    }
    return true;
  }

  // ---- LRU eviction --------------------------------------------------------------------------
  struct HeapItem {
    uint64_t priority;
    int32_t node;
  };
  // Python heapq over (priority, node) tuples: an item is "less" only on a strictly smaller priority.
  static bool heap_less(const HeapItem &a, const HeapItem &b) { return a.priority < b.priority; }

  // heapq._siftdown / _siftup / heapify / heappop / heappush, restated so ties resolve identically.
  static void sift_down(std::vector<HeapItem> &h, size_t start, size_t pos) {
    HeapItem item = h[pos];
    while (pos > start) {
      size_t parent = (pos - 1) >> 1;
      if (heap_less(item, h[parent])) {
        h[pos] = h[parent];
        pos = parent;
        continue;
      }
      break;
    }
    h[pos] = item;
  }
  static void sift_up(std::vector<HeapItem> &h, size_t pos) {
    size_t end = h.size(), start = pos;
    HeapItem item = h[pos];
    size_t child = 2 * pos + 1;
    while (child < end) {
      size_t right = child + 1;
      if (right < end && !heap_less(h[child], h[right])) child = right;
      h[pos] = h[child];
      pos = child;
      child = 2 * pos + 1;
    }
    h[pos] = item;
    sift_down(h, start, pos);
  }
  static void heapify(std::vector<HeapItem> &h) {
    for (size_t i = h.size() / 2; i-- > 0;) sift_up(h, i);
  }
  static HeapItem heappop(std::vector<HeapItem> &h) {
    HeapItem last = h.back();
    h.pop_back();
    if (!h.empty()) {
      HeapItem ret = h[0];
      h[0] = last;
      sift_up(h, 0);
      return ret;
    }
    return last;
  }
  static void heappush(std::vector<HeapItem> &h, HeapItem it) {
    h.push_back(it);
    sift_down(h, 0, h.size() - 1);
  }

  void collect_leaves(std::vector<int32_t> &out) const {
    std::vector<int32_t> stack{root};
    while (!stack.empty()) {
      int32_t cur = stack.back();
      stack.pop_back();
      const Node &n = nodes[cur];
      if (n.children.empty()) {
        out.push_back(cur);
      } else {
        stack.insert(stack.end(), n.children.begin(), n.children.end());
      }
    }
  }

  int64_t evict(int64_t num_tokens) {
    std::vector<int32_t> leaves;
    collect_leaves(leaves);
    std::vector<HeapItem> heap;
    heap.reserve(leaves.size());
    for (int32_t l : leaves) heap.push_back({nodes[l].last_access, l});
    heapify(heap);
    int64_t evicted = 0;
    while (evicted < num_tokens && !heap.empty()) {
      HeapItem it = heappop(heap);
      int32_t x = it.node;
      if (x == root) break;
      if (nodes[x].lock_ref > 0) continue;
      free_slots(nodes[x].value.data(), int64_t(nodes[x].value.size()), /*check=*/false);
      evicted += int64_t(nodes[x].value.size());
      int32_t parent = nodes[x].parent;
      std::vector<int32_t> &pc = nodes[parent].children;
      pc.erase(std::find(pc.begin(), pc.end(), x));
      evictable -= int64_t(nodes[x].key.size());
      drop_node(x);
      if (pc.empty()) heappush(heap, {nodes[parent].last_access, parent});
    }
    return evicted;
  }

  // ---- allocator -----------------------------------------------------------------------------
  int64_t available_units() const { return int64_t(free_units.size() - free_head) + int64_t(release_units.size()); }
  int64_t available() const { return available_units() * page; }

  void merge_and_sort() {
    if (release_units.empty()) return;
    std::vector<int64_t> merged(free_units.begin() + std::ptrdiff_t(free_head), free_units.end());
    merged.insert(merged.end(), release_units.begin(), release_units.end());
    std::sort(merged.begin(), merged.end());
    free_units.swap(merged);
    free_head = 0;
    release_units.clear();
  }

  bool alloc(int64_t n, int64_t *out) {
    int64_t units = page == 1 ? n : (n + page - 1) / page;
    if (units > int64_t(free_units.size() - free_head)) merge_and_sort();
    if (units > int64_t(free_units.size() - free_head)) return false;
    const int64_t *u = free_units.data() + free_head;
    if (page == 1) {
      std::memcpy(out, u, size_t(n) * sizeof(int64_t));
    } else {
      int64_t t = 0;
      for (int64_t i = 0; i < units && t < n; ++i) {
        const int64_t base = u[i] * page;
        for (int64_t o = 0; o < page && t < n; ++o) out[t++] = base + o;
      }
    }
    for (int64_t i = 0; i < units; ++i) unit_free[size_t(u[i])] = 0;
    free_head += size_t(units);
    if (free_head == free_units.size()) {
      free_units.clear();
      free_head = 0;
    }
    return true;
  }

  // Returns false when a slot is out of range or already free (check == true).
  bool free_slots(const int64_t *s, int64_t n, bool check) {
    if (n <= 0) return true;
    if (page == 1) {
      if (check) {
        for (int64_t i = 0; i < n; ++i)
          if (s[i] < 1 || s[i] > num_pages || unit_free[size_t(s[i])]) return false;
      }
      for (int64_t i = 0; i < n; ++i) unit_free[size_t(s[i])] = 1;
      release_units.insert(release_units.end(), s, s + n);
      return true;
    }
    // unique pages, ascending (torch.unique(free_index // page_size)); the slots of a page come as runs, so
    // adjacent repeats are dropped first and only the distinct pages are sorted
    std::vector<int64_t> pages;
    pages.reserve(static_cast<size_t>(n / page + 2));
    for (int64_t i = 0; i < n; ++i) {
      const int64_t p = s[i] >= 0 ? s[i] / page : -1;
      if (pages.empty() || pages.back() != p) pages.push_back(p);
    }
    std::sort(pages.begin(), pages.end());
    pages.erase(std::unique(pages.begin(), pages.end()), pages.end());
    if (check) {
      for (int64_t p : pages)
        if (p < 1 || p > num_pages || unit_free[size_t(p)]) return false;
    }
    for (int64_t p : pages) unit_free[size_t(p)] = 1;
    release_units.insert(release_units.end(), pages.begin(), pages.end());
    return true;
  }
};

}  // namespace qe

struct qe_index {
  qe::Index ix;
};

using qe::fail;

extern "C" {

const char *qe_last_error(void) { return qe::last_error().c_str(); }

int qe_index_create(int64_t capacity_tokens, int32_t page_size, qe_index **out) {
  QE_CHECK_ARG(out != nullptr, "qe_index_create: out is null");
  QE_CHECK_ARG(page_size >= 1, "qe_index_create: page_size must be >= 1 (got %d)", page_size);
  QE_CHECK_ARG(capacity_tokens >= page_size, "qe_index_create: capacity %lld below one page",
               (long long)capacity_tokens);
  qe_index *h = new (std::nothrow) qe_index();
  if (!h) return fail(QE_ERR_NOMEM, "qe_index_create: out of host memory");
  try {
    h->ix.page = page_size;
    h->ix.num_pages = capacity_tokens / page_size;
    h->ix.capacity = h->ix.num_pages * page_size;
    h->ix.reset_tree();
    h->ix.reset_alloc();
  } catch (const std::bad_alloc &) {
    delete h;
    return fail(QE_ERR_NOMEM, "qe_index_create: out of host memory");
  }
  *out = h;
  return qe::ok();
}

int qe_index_destroy(qe_index *ix) {
  delete ix;
  return qe::ok();
}

int qe_index_clear(qe_index *ix) {
  QE_CHECK_ARG(ix, "qe_index_clear: null index");
  ix->ix.reset_tree();
  ix->ix.reset_alloc();
  return qe::ok();
}

int qe_index_match(qe_index *ix, const int64_t *key, int64_t n, int64_t *out_len, int64_t *out_slots,
                   uint64_t *out_node) {
  QE_CHECK_ARG(ix && out_len && out_node, "qe_index_match: null argument");
  QE_CHECK_ARG(n >= 0, "qe_index_match: negative length");
  QE_CHECK_ARG(n == 0 || (key && out_slots), "qe_index_match: null key or output");
  try {
    ix->ix.match(key, n, out_len, out_slots, out_node);
  } catch (const std::bad_alloc &) {
    return fail(QE_ERR_NOMEM, "qe_index_match: out of host memory");
  }
  return qe::ok();
}

int qe_index_lock(qe_index *ix, uint64_t node) {
  QE_CHECK_ARG(ix, "qe_index_lock: null index");
  int32_t id = ix->ix.resolve(node);
  if (id < 0 || id == ix->ix.root) return fail(QE_ERR_INVALID, "qe_index_lock: stale or invalid node handle");
  ix->ix.lock(id);
  return qe::ok();
}

int qe_index_unlock(qe_index *ix, uint64_t node) {
  QE_CHECK_ARG(ix, "qe_index_unlock: null index");
  int32_t id = ix->ix.resolve(node);
  if (id < 0 || id == ix->ix.root) return fail(QE_ERR_INVALID, "qe_index_unlock: stale or invalid node handle");
  if (!ix->ix.unlock(id)) return fail(QE_ERR_STATE, "qe_index_unlock: node path holds no lock");
  return qe::ok();
}

int qe_index_insert(qe_index *ix, const int64_t *key, const int64_t *slots, int64_t n, int64_t *out_present) {
  QE_CHECK_ARG(ix && out_present, "qe_index_insert: null argument");
  QE_CHECK_ARG(n >= 0, "qe_index_insert: negative length");
  QE_CHECK_ARG(n == 0 || (key && slots), "qe_index_insert: null key or slots");
  {  // the stored slots are freed by eviction later without a check: reject out-of-range ones here, before
     // the tree changes (page 0, slots 0 .. page_size - 1, is padding)
    const qe::Index &x = ix->ix;
    const int64_t stored = x.aligned(n), lo = x.page, hi = (x.num_pages + 1) * x.page;
    for (int64_t i = 0; i < stored; ++i)
      if (slots[i] < lo || slots[i] >= hi)
        return fail(QE_ERR_INVALID, "qe_index_insert: slot %lld at position %lld outside [%lld, %lld)",
                    (long long)slots[i], (long long)i, (long long)lo, (long long)hi);
  }
  try {
    *out_present = ix->ix.insert(key, slots, n);
  } catch (const std::bad_alloc &) {
    return fail(QE_ERR_NOMEM, "qe_index_insert: out of host memory");
  }
  return qe::ok();
}

int qe_index_evict(qe_index *ix, int64_t num_tokens, int64_t *out_evicted) {
  QE_CHECK_ARG(ix && out_evicted, "qe_index_evict: null argument");
  try {
    *out_evicted = num_tokens > 0 ? ix->ix.evict(num_tokens) : 0;
  } catch (const std::bad_alloc &) {
    return fail(QE_ERR_NOMEM, "qe_index_evict: out of host memory");
  }
  return qe::ok();
}

int qe_index_alloc(qe_index *ix, int64_t n, int64_t *out_slots, int32_t *out_ok) {
  QE_CHECK_ARG(ix && out_ok, "qe_index_alloc: null argument");
  QE_CHECK_ARG(n >= 0, "qe_index_alloc: negative size");
  QE_CHECK_ARG(n == 0 || out_slots, "qe_index_alloc: null output");
  try {
    *out_ok = ix->ix.alloc(n, out_slots) ? 1 : 0;
  } catch (const std::bad_alloc &) {
    return fail(QE_ERR_NOMEM, "qe_index_alloc: out of host memory");
  }
  return qe::ok();
}

int qe_index_free(qe_index *ix, const int64_t *slots, int64_t n) {
  QE_CHECK_ARG(ix, "qe_index_free: null index");
  QE_CHECK_ARG(n >= 0 && (n == 0 || slots), "qe_index_free: bad slots");
  try {
    if (!ix->ix.free_slots(slots, n, /*check=*/true))
      return fail(QE_ERR_STATE, "qe_index_free: slot out of range or already free");
  } catch (const std::bad_alloc &) {
    return fail(QE_ERR_NOMEM, "qe_index_free: out of host memory");
  }
  return qe::ok();
}

int qe_index_shuffle_free(qe_index *ix, uint64_t seed) {
  QE_CHECK_ARG(ix, "qe_index_shuffle_free: null index");
  qe::Index &x = ix->ix;
  // Fisher-Yates over the not-yet-allocated head of the free list, splitmix64 as the generator
  uint64_t state = seed;
  auto next = [&state]() {
    uint64_t z = (state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  };
  int64_t *u = x.free_units.data() + x.free_head;
  int64_t n = int64_t(x.free_units.size() - x.free_head);
  for (int64_t i = n - 1; i > 0; --i) std::swap(u[i], u[int64_t(next() % uint64_t(i + 1))]);
  return qe::ok();
}

int qe_index_usage(qe_index *ix, int64_t out[4]) {
  QE_CHECK_ARG(ix && out, "qe_index_usage: null argument");
  out[0] = ix->ix.available();
  out[1] = ix->ix.evictable;
  out[2] = ix->ix.protected_;
  out[3] = ix->ix.live_nodes;
  return qe::ok();
}

}  // extern "C"
