// Expert-cache policy (host code): which expert occupies which HBM slot. The same decisions as the reference's
// c/src/cache.c (cl_cache_*): plain LRU, or W-TinyLFU -- an admission window in front of a segmented LRU (probation +
// protected) whose admission compares 4-bit count-min-sketch frequencies -- optionally with the window size tuned by hill
// climbing on the hit rate; plus a staging area for prefetched experts, so a prefetch never evicts something the policy
// keeps. Slot numbers, list orders, sketch hashing and aging follow the reference step for step, so a replay of the same
// operations gives the same results and the same slots (the tests check this against the reference's own code).
//
// The policy holds no expert data; the device store (store.cu) owns the HBM slots and the copies.
#include <cstdint>
#include <cstdlib>
#include <new>
#include <vector>

#include "../../include/clb200.h"

namespace {

enum Seg : int { FREE = 0, WINDOW = 1, PROBATION = 2, PROTECTED = 3, STAGE = 4 };
constexpr uint32_t NO_KEY = UINT32_MAX;

// splitmix64 finaliser: the sketch's hash (cache.c:30)
uint64_t mix(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

struct Slot {
  int prev = -1, next = -1;
  uint32_t key = NO_KEY;
  int seg = FREE;
  int pins = 0;
};

struct Ring {   // intrusive doubly linked list over slot indices; head = most recent
  int head = -1, tail = -1;
  uint32_t n = 0;
};

}  // namespace

struct clb200_cache {
  int policy;
  uint32_t cap, stage_cap, total, universe, win_cap, main_cap, prot_cap;
  std::vector<Slot> slot;
  std::vector<int> where;   // key -> slot, or -1
  Ring seg[5];
  // 4-bit count-min sketch, 4 rows of `width` counters, two counters a byte (cache.c:31-51)
  std::vector<uint8_t> cms;
  uint32_t width = 0;
  uint64_t adds = 0, sample = 0;
  // adaptive window (cache.c:173-183)
  uint64_t hc_period = 0, hc_acc = 0, hc_hit = 0;
  double hc_prev = -1.0;
  int hc_dir = 1;
  clb200_cache_stats st{};

  uint32_t cached() const { return seg[WINDOW].n + seg[PROBATION].n + seg[PROTECTED].n; }

  // -- lists
  void unlink(int i) {
    Slot &s = slot[i];
    Ring &r = seg[s.seg];
    if (s.prev >= 0) slot[s.prev].next = s.next; else r.head = s.next;
    if (s.next >= 0) slot[s.next].prev = s.prev; else r.tail = s.prev;
    --r.n;
    s.prev = s.next = -1;
  }
  void push_front(int i, int to) {
    Slot &s = slot[i];
    Ring &r = seg[to];
    s.seg = to;
    s.prev = -1;
    s.next = r.head;
    if (r.head >= 0) slot[r.head].prev = i; else r.tail = i;
    r.head = i;
    ++r.n;
  }
  void move_front(int i, int to) { unlink(i); push_front(i, to); }
  // least recent unpinned slot of a list, skipping `skip`
  int oldest_unpinned(int s, int skip) const {
    for (int i = seg[s].tail; i >= 0; i = slot[i].prev)
      if (!slot[i].pins && i != skip) return i;
    return -1;
  }
  void drop(int i) {   // back to the free list
    Slot &s = slot[i];
    if (s.seg != FREE) unlink(i);
    if (s.key != NO_KEY) where[s.key] = -1;
    s.key = NO_KEY;
    s.pins = 0;
    push_front(i, FREE);
  }
  int take_free() {
    const int i = seg[FREE].head;
    if (i >= 0) unlink(i);
    return i;
  }

  // -- sketch
  uint32_t cell(uint32_t key, int row) const {
    return static_cast<uint32_t>(mix((static_cast<uint64_t>(key) << 3) ^ static_cast<uint64_t>(row + 1) * 0x2545f4914f6cdd1dull)) & (width - 1);
  }
  uint32_t get(uint32_t i, int row) const {
    const uint8_t b = cms[static_cast<size_t>(row) * width / 2 + i / 2];
    return (i & 1) ? b >> 4 : b & 15u;
  }
  void put(uint32_t i, int row, uint32_t v) {
    uint8_t &b = cms[static_cast<size_t>(row) * width / 2 + i / 2];
    b = (i & 1) ? static_cast<uint8_t>((b & 0x0f) | (v << 4)) : static_cast<uint8_t>((b & 0xf0) | v);
  }
  uint32_t freq(uint32_t key) const {
    uint32_t m = 15;
    for (int r = 0; r < 4; ++r) {
      const uint32_t v = get(cell(key, r), r);
      if (v < m) m = v;
    }
    return m;
  }
  void count(uint32_t key) {   // conservative update; all counters halve every `sample` additions
    uint32_t c[4], v[4], m = 15;
    for (int r = 0; r < 4; ++r) {
      c[r] = cell(key, r);
      v[r] = get(c[r], r);
      if (v[r] < m) m = v[r];
    }
    if (m < 15)
      for (int r = 0; r < 4; ++r)
        if (v[r] == m) put(c[r], r, m + 1);
    if (++adds >= sample) {
      for (uint8_t &b : cms) b = static_cast<uint8_t>((b >> 1) & 0x77);
      adds = 0;
      ++st.aging_resets;
    }
  }

  // -- policy
  // Evicts until the cache holds at most `cap` experts; false when everything evictable is pinned.
  bool make_room(int keep) {
    while (cached() > cap) {
      if (policy == CLB200_LRU) {
        const int v = oldest_unpinned(WINDOW, keep);
        if (v < 0) return false;
        ++st.evictions;
        drop(v);
        continue;
      }
      if (seg[WINDOW].n > win_cap) {   // the window's oldest tries to enter the main segment
        const int cand = oldest_unpinned(WINDOW, keep);
        if (cand >= 0) {
          move_front(cand, PROBATION);
          if (seg[PROBATION].n + seg[PROTECTED].n > main_cap) {
            int victim = oldest_unpinned(PROBATION, -1);
            if (victim < 0) victim = cand;
            const int loser = (victim != cand && freq(slot[cand].key) >= freq(slot[victim].key)) ? victim : cand;
            if (loser == cand) ++st.admit_rejects;
            ++st.evictions;
            drop(loser);
          }
          continue;
        }
      }
      int v = oldest_unpinned(PROBATION, keep);
      if (v < 0) v = oldest_unpinned(PROTECTED, keep);
      if (v < 0) v = oldest_unpinned(WINDOW, keep);
      if (v < 0) return false;
      ++st.evictions;
      drop(v);
    }
    return true;
  }
  void touch(int i) {
    switch (slot[i].seg) {
      case WINDOW: move_front(i, WINDOW); break;
      case PROTECTED: move_front(i, PROTECTED); break;
      case PROBATION:
        if (policy == CLB200_LRU) break;
        move_front(i, PROTECTED);   // a second hit promotes; the protected segment's overflow goes back to probation
        while (seg[PROTECTED].n > prot_cap) {
          const int d = oldest_unpinned(PROTECTED, i);
          if (d < 0) break;
          move_front(d, PROBATION);
        }
        break;
      default: break;
    }
  }
  void set_window(uint32_t w) {
    const uint32_t hi = cap > 1 ? cap - 1 : 1;
    if (w < 1) w = 1;
    if (w > hi) w = hi;
    win_cap = w;
    main_cap = cap - w;
    prot_cap = main_cap * 4 / 5;
  }
  void climb(int hit) {   // adaptive policy: every period, keep moving the window the way that did not hurt
    ++hc_acc;
    hc_hit += static_cast<uint64_t>(hit);
    if (hc_acc < hc_period) return;
    const double rate = static_cast<double>(hc_hit) / static_cast<double>(hc_acc);
    if (hc_prev >= 0) {
      if (rate < hc_prev - 0.002) hc_dir = -hc_dir;
      const uint32_t step = cap / 20 ? cap / 20 : 1;
      set_window(hc_dir > 0 ? win_cap + step : (win_cap > step ? win_cap - step : 1));
    }
    hc_prev = rate;
    hc_acc = hc_hit = 0;
  }
};

extern "C" {

clb200_cache *clb200_cache_new(uint32_t cache_slots, uint32_t stage_slots, uint32_t universe, int policy, uint32_t window_pct) {
  if (cache_slots == 0 || universe == 0 || policy < CLB200_LRU || policy > CLB200_ADAPTIVE) return nullptr;
  clb200_cache *c = new (std::nothrow) clb200_cache();
  if (!c) return nullptr;
  try {
    c->policy = policy;
    c->cap = cache_slots;
    c->stage_cap = stage_slots;
    c->universe = universe;
    c->total = cache_slots + stage_slots + 1;   // one spare: an insert comes before the eviction it causes
    if (policy == CLB200_ADAPTIVE) {
      c->hc_period = static_cast<uint64_t>(cache_slots) * 8 > 500 ? static_cast<uint64_t>(cache_slots) * 8 : 500;
      if (!window_pct) window_pct = 10;
    }
    if (policy == CLB200_LRU) {
      c->win_cap = cache_slots;
      c->main_cap = 0;
    } else {
      if (!window_pct || window_pct > 90) window_pct = 1;
      c->win_cap = cache_slots * window_pct / 100 ? cache_slots * window_pct / 100 : 1;
      if (c->win_cap >= cache_slots) c->win_cap = cache_slots > 1 ? cache_slots - 1 : 1;
      c->main_cap = cache_slots - c->win_cap;
    }
    c->prot_cap = c->main_cap * 4 / 5;
    c->slot.resize(c->total);
    c->where.assign(universe, -1);
    uint32_t w = 256;
    while (w < universe * 4) w <<= 1;
    c->width = w;
    c->cms.assign(static_cast<size_t>(4) * w / 2, 0);
    c->sample = static_cast<uint64_t>(cache_slots) * 10 > 1000 ? static_cast<uint64_t>(cache_slots) * 10 : 1000;
    for (uint32_t i = 0; i < c->total; ++i) c->push_front(static_cast<int>(i), FREE);
  } catch (...) {
    delete c;
    return nullptr;
  }
  return c;
}

void clb200_cache_free(clb200_cache *c) { delete c; }
uint32_t clb200_cache_total_slots(const clb200_cache *c) { return c->total; }
int clb200_cache_find(const clb200_cache *c, uint32_t key) { return key < c->universe ? c->where[key] : -1; }
int clb200_cache_segment(const clb200_cache *c, int slot) { return c->slot[slot].seg; }
uint32_t clb200_cache_slot_key(const clb200_cache *c, int slot) { return c->slot[slot].key; }
uint32_t clb200_cache_count(const clb200_cache *c) { return c->cached(); }
uint32_t clb200_cache_freq(const clb200_cache *c, uint32_t key) { return c->freq(key); }
void clb200_cache_pin(clb200_cache *c, int slot) { ++c->slot[slot].pins; }
void clb200_cache_unpin(clb200_cache *c, int slot) {
  if (c->slot[slot].pins > 0) --c->slot[slot].pins;
}
void clb200_cache_abandon(clb200_cache *c, int slot) { c->drop(slot); }
clb200_cache_stats clb200_cache_get_stats(const clb200_cache *c) {
  clb200_cache_stats s = c->st;
  s.window_slots = c->win_cap;
  return s;
}

int clb200_cache_access(clb200_cache *c, uint32_t key, int *slot) {
  *slot = -1;
  if (key >= c->universe) return -1;
  c->count(key);
  const int i = c->where[key];
  if (i >= 0 && c->slot[i].seg == STAGE) {   // a prefetched expert was wanted: it joins the cache
    ++c->st.stage_hits;
    if (c->policy == CLB200_ADAPTIVE) c->climb(1);
    c->move_front(i, WINDOW);
    ++c->slot[i].pins;
    c->make_room(i);
    *slot = i;
    return 2;
  }
  if (i >= 0) {
    ++c->st.hits;
    if (c->policy == CLB200_ADAPTIVE) c->climb(1);
    c->touch(i);
    ++c->slot[i].pins;
    *slot = i;
    return 1;
  }
  ++c->st.misses;
  if (c->policy == CLB200_ADAPTIVE) c->climb(0);
  const int n = c->take_free();
  if (n < 0) return -1;
  c->slot[n].key = key;
  c->slot[n].pins = 1;
  c->where[key] = n;
  c->push_front(n, WINDOW);
  ++c->st.inserts;
  if (!c->make_room(n)) {   // everything else is pinned: the over-capacity entry is not kept
    c->drop(n);
    return -1;
  }
  *slot = n;
  return 0;
}

int clb200_cache_stage(clb200_cache *c, uint32_t key) {
  if (key >= c->universe || c->where[key] >= 0 || c->stage_cap == 0) return -1;
  if (c->seg[STAGE].n >= c->stage_cap) {   // the oldest unclaimed prefetch makes way
    const int old = c->oldest_unpinned(STAGE, -1);
    if (old < 0) return -1;
    ++c->st.stage_wasted;
    c->drop(old);
  }
  const int n = c->take_free();
  if (n < 0) return -1;
  c->slot[n].key = key;
  c->slot[n].pins = 1;
  c->where[key] = n;
  c->push_front(n, STAGE);
  ++c->st.stage_inserts;
  return n;
}

}  // extern "C"
