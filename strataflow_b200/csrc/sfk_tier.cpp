// sfk_tier.cpp -- the bounded expert tier's slot pool and predictor (host).
#include "sfk_tier.h"

#include <algorithm>
#include <numeric>

namespace sfk {

SlotPool::SlotPool(uint32_t n_slots) : n_slots_(n_slots) { clear(); }

SlotPool::SlotPool(uint32_t n_slots, uint32_t n_layer, uint32_t n_expert, uint32_t n_expert_used)
    : n_slots_(n_slots) {
  clear();
  if (n_layer == 0 || n_expert == 0) return;  // degenerate shape: the global pool
  stratified_ = true;
  n_layer_ = n_layer;
  n_expert_ = n_expert;
  n_expert_used_ = n_expert_used == 0 ? 1 : n_expert_used;
  layers_.assign(n_layer_, LayerState{});
  cap_.assign(n_layer_, 0);
  recompute_caps({});
}

void SlotPool::clear() {
  map_.clear();
  lru_.clear();
  for (LayerState& ls : layers_) {
    ls.lru.clear();
    ls.resident = 0;
  }
  free_slots_.clear();
  for (uint32_t i = 0; i < n_slots_; ++i) free_slots_.push_back(n_slots_ - 1 - i);  // slots 0, 1, 2, ... first
  pinned_.assign(n_slots_, 0);
  n_pinned_ = 0;
}

// Per-layer capacities (weight_store.cpp:44-119): every layer gets the floor
// min(n_expert_used, n_expert) (shrunk to n_slots / n_layer, at least 1, when
// the budget cannot afford it), then the spare slots go one at a time to the
// layers in descending weight order (stable by index), cycling until the
// budget is spent or every layer holds all its experts.
void SlotPool::recompute_caps(const std::vector<uint64_t>& weights) {
  if (!stratified_) return;
  uint32_t floor = std::min(n_expert_used_, n_expert_);
  if (floor == 0) floor = 1;
  if ((uint64_t)floor * n_layer_ > n_slots_) {
    floor = n_slots_ / n_layer_;
    if (floor == 0) floor = 1;
  }
  const uint32_t ceil = n_expert_;
  uint64_t used = 0;
  for (uint32_t l = 0; l < n_layer_; ++l) {
    cap_[l] = std::min(floor, ceil);
    used += cap_[l];
  }
  uint64_t spare = used < n_slots_ ? n_slots_ - used : 0;
  if (spare == 0) return;
  std::vector<uint32_t> order(n_layer_);
  std::iota(order.begin(), order.end(), 0u);
  if (weights.size() == n_layer_)
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return weights[a] > weights[b]; });
  bool progress = true;
  while (spare > 0 && progress) {
    progress = false;
    for (uint32_t i = 0; i < n_layer_ && spare > 0; ++i) {
      const uint32_t l = order[i];
      if (cap_[l] < ceil) {
        ++cap_[l];
        --spare;
        progress = true;
      }
    }
  }
}

void SlotPool::set_layer_weights(const std::vector<uint64_t>& weights) {
  if (!stratified_ || weights.size() != n_layer_) return;
  recompute_caps(weights);
}

uint32_t SlotPool::layer_capacity(uint32_t layer) const {
  if (!stratified_) return n_slots_;
  return layer < cap_.size() ? cap_[layer] : 0;
}

bool SlotPool::has_free_slot() const {
  if (!stratified_) return !free_slots_.empty() || map_.size() < n_slots_;
  if (!free_slots_.empty()) return true;
  for (uint32_t l = 0; l < n_layer_; ++l)
    if (layers_[l].resident < cap_[l]) return true;
  return false;
}

bool SlotPool::has_free_slot_in_layer(uint32_t layer) const {
  if (!stratified_) return has_free_slot();
  if (layer >= n_layer_) return false;
  return !free_slots_.empty() && layers_[layer].resident < cap_[layer];
}

bool SlotPool::resident(uint32_t layer, uint32_t expert) const { return map_.count(key(layer, expert)) != 0; }

uint32_t SlotPool::slot_of(uint32_t layer, uint32_t expert) const {
  auto it = map_.find(key(layer, expert));
  return it == map_.end() ? NONE : it->second.slot;
}

void SlotPool::pin(uint32_t slot) {
  if (slot < n_slots_ && !pinned_[slot]) {
    pinned_[slot] = 1;
    ++n_pinned_;
  }
}

void SlotPool::unpin_all() {
  std::fill(pinned_.begin(), pinned_.end(), 0);
  n_pinned_ = 0;
}

std::list<uint64_t>::iterator SlotPool::victim(std::list<uint64_t>& lru) {
  for (auto it = lru.end(); it != lru.begin();) {
    --it;
    if (!pinned_[map_.at(*it).slot]) return it;
  }
  return lru.end();
}

uint32_t SlotPool::evict(std::list<uint64_t>& lru, std::list<uint64_t>::iterator v) {
  const uint64_t k = *v;
  auto mit = map_.find(k);
  const uint32_t slot = mit->second.slot;
  map_.erase(mit);
  lru.erase(v);
  if (stratified_) --layers_[key_layer(k)].resident;
  ++stats_.evictions;
  return slot;
}

uint32_t SlotPool::acquire(uint32_t layer, uint32_t expert, bool* miss) {
  if (miss) *miss = false;
  if (n_slots_ == 0) return NONE;
  if (stratified_ && layer >= n_layer_) layer = 0;  // (weight_store.h:216)
  const uint64_t k = key(layer, expert);
  auto it = map_.find(k);
  if (it != map_.end()) {  // hit: most recent in its list
    ++stats_.hits;
    std::list<uint64_t>& lru = stratified_ ? layers_[layer].lru : lru_;
    lru.splice(lru.begin(), lru, it->second.it);
    return it->second.slot;
  }
  uint32_t slot = NONE;
  if (!stratified_) {
    if (!free_slots_.empty()) {
      slot = free_slots_.back();
      free_slots_.pop_back();
    } else {
      auto v = victim(lru_);
      if (v == lru_.end()) return NONE;
      slot = evict(lru_, v);
    }
    lru_.push_front(k);
    map_[k] = Entry{slot, lru_.begin()};
  } else {
    LayerState& ls = layers_[layer];
    std::list<uint64_t>::iterator v;
    if (ls.resident < cap_[layer] && !free_slots_.empty()) {
      slot = free_slots_.back();
      free_slots_.pop_back();
    } else if ((v = victim(ls.lru)) != ls.lru.end()) {  // the layer's own LRU victim
      slot = evict(ls.lru, v);
    } else if (!free_slots_.empty()) {
      slot = free_slots_.back();
      free_slots_.pop_back();
    } else {
      // the most over-capacity layer that has an unpinned resident
      int64_t worst = 0;
      int donor = -1;
      for (uint32_t l = 0; l < n_layer_; ++l) {
        if (victim(layers_[l].lru) == layers_[l].lru.end()) continue;
        const int64_t over = (int64_t)layers_[l].resident - (int64_t)cap_[l];
        if (donor < 0 || over > worst) {
          worst = over;
          donor = (int)l;
        }
      }
      if (donor < 0) return NONE;
      std::list<uint64_t>& dl = layers_[donor].lru;
      slot = evict(dl, victim(dl));
    }
    ls.lru.push_front(k);
    map_[k] = Entry{slot, ls.lru.begin()};
    ++ls.resident;
  }
  ++stats_.misses;
  if (miss) *miss = true;
  return slot;
}

ExpertPredictor::ExpertPredictor(uint32_t n_layer, uint32_t n_expert)
    : n_layer_(n_layer), n_expert_(n_expert), freq_((size_t)n_layer * n_expert, 0) {}

void ExpertPredictor::observe(uint32_t layer, uint32_t expert) {
  if (layer < n_layer_ && expert < n_expert_) ++freq_[(size_t)layer * n_expert_ + expert];
  if (std::find(last_.begin(), last_.end(), expert) != last_.end()) ++confirmed_;
}

std::vector<uint32_t> ExpertPredictor::predict(uint32_t layer, uint32_t k) {
  std::vector<uint32_t> out;
  if (layer >= n_layer_ || k == 0) return out;
  const uint64_t* f = freq_.data() + (size_t)layer * n_expert_;
  std::vector<uint32_t> idx(n_expert_);
  std::iota(idx.begin(), idx.end(), 0u);
  const size_t take = std::min<size_t>(k, idx.size());
  std::partial_sort(idx.begin(), idx.begin() + take, idx.end(),
                    [&](uint32_t a, uint32_t b) { return f[a] != f[b] ? f[a] > f[b] : a < b; });
  out.assign(idx.begin(), idx.begin() + take);
  predicted_ += out.size();
  last_ = out;
  return out;
}

std::vector<uint64_t> ExpertPredictor::layer_activity() const {
  std::vector<uint64_t> out(n_layer_, 0);
  for (uint32_t l = 0; l < n_layer_; ++l)
    for (uint32_t e = 0; e < n_expert_; ++e) out[l] += freq_[(size_t)l * n_expert_ + e];
  return out;
}

}  // namespace sfk

// ---------------------------------------------------------------------------
// C ABI (include/sfk.h): the pool and the predictor for host-side callers
// ---------------------------------------------------------------------------
#include <new>

#include "sfk.h"

namespace sfk {
void set_last_error(const char* msg);
}

struct sfk_pool {
  sfk::SlotPool pool;
};
struct sfk_predictor {
  sfk::ExpertPredictor pred;
};

extern "C" {

sfk_status sfk_pool_create(uint32_t n_slots, uint32_t n_layer, uint32_t n_expert, uint32_t n_expert_used,
                           sfk_pool** out) {
  if (!out) {
    sfk::set_last_error("sfk_pool_create: null out");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  *out = n_layer == 0 ? new (std::nothrow) sfk_pool{sfk::SlotPool(n_slots)}
                      : new (std::nothrow) sfk_pool{sfk::SlotPool(n_slots, n_layer, n_expert, n_expert_used)};
  if (!*out) {
    sfk::set_last_error("sfk_pool_create: host allocation failed");
    return SFK_ERR_OUT_OF_MEMORY;
  }
  return SFK_OK;
}

void sfk_pool_free(sfk_pool* p) { delete p; }

int64_t sfk_pool_acquire(sfk_pool* p, uint32_t layer, uint32_t expert, int32_t* miss_out) {
  if (!p) return -1;
  bool miss = false;
  const uint32_t s = p->pool.acquire(layer, expert, &miss);
  if (miss_out) *miss_out = miss ? 1 : 0;
  return s == sfk::SlotPool::NONE ? -1 : (int64_t)s;
}

int32_t sfk_pool_resident(const sfk_pool* p, uint32_t layer, uint32_t expert) {
  return p && p->pool.resident(layer, expert) ? 1 : 0;
}

int32_t sfk_pool_stratified(const sfk_pool* p) { return p && p->pool.stratified() ? 1 : 0; }

uint32_t sfk_pool_layer_capacity(const sfk_pool* p, uint32_t layer) { return p ? p->pool.layer_capacity(layer) : 0; }

int32_t sfk_pool_has_free_slot_in_layer(const sfk_pool* p, uint32_t layer) {
  return p && p->pool.has_free_slot_in_layer(layer) ? 1 : 0;
}

sfk_status sfk_pool_set_layer_weights(sfk_pool* p, const uint64_t* w, uint32_t n_layer) {
  if (!p || (!w && n_layer)) {
    sfk::set_last_error("sfk_pool_set_layer_weights: null argument");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  p->pool.set_layer_weights(std::vector<uint64_t>(w, w + n_layer));
  return SFK_OK;
}

sfk_status sfk_pool_pin(sfk_pool* p, uint32_t slot) {
  if (!p || slot >= p->pool.n_slots()) {
    sfk::set_last_error("sfk_pool_pin: no such slot");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  p->pool.pin(slot);
  return SFK_OK;
}

sfk_status sfk_pool_unpin_all(sfk_pool* p) {
  if (!p) {
    sfk::set_last_error("sfk_pool_unpin_all: null pool");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  p->pool.unpin_all();
  return SFK_OK;
}

sfk_status sfk_pool_stats(const sfk_pool* p, uint64_t out[3]) {
  if (!p || !out) {
    sfk::set_last_error("sfk_pool_stats: null argument");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  out[0] = p->pool.stats().hits;
  out[1] = p->pool.stats().misses;
  out[2] = p->pool.stats().evictions;
  return SFK_OK;
}

sfk_status sfk_predictor_create(uint32_t n_layer, uint32_t n_expert, sfk_predictor** out) {
  if (!out) {
    sfk::set_last_error("sfk_predictor_create: null out");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  *out = new (std::nothrow) sfk_predictor{sfk::ExpertPredictor(n_layer, n_expert)};
  if (!*out) {
    sfk::set_last_error("sfk_predictor_create: host allocation failed");
    return SFK_ERR_OUT_OF_MEMORY;
  }
  return SFK_OK;
}

void sfk_predictor_free(sfk_predictor* p) { delete p; }

sfk_status sfk_predictor_observe(sfk_predictor* p, uint32_t layer, uint32_t expert) {
  if (!p) {
    sfk::set_last_error("sfk_predictor_observe: null predictor");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  p->pred.observe(layer, expert);
  return SFK_OK;
}

uint32_t sfk_predictor_predict(sfk_predictor* p, uint32_t layer, uint32_t k, uint32_t* out) {
  if (!p || !out) return 0;
  const std::vector<uint32_t> v = p->pred.predict(layer, k);
  std::copy(v.begin(), v.end(), out);
  return (uint32_t)v.size();
}

double sfk_predictor_accuracy(const sfk_predictor* p) { return p ? p->pred.accuracy() : 0.0; }

sfk_status sfk_predictor_layer_activity(const sfk_predictor* p, uint64_t* out, uint32_t n_layer) {
  if (!p || !out) {
    sfk::set_last_error("sfk_predictor_layer_activity: null argument");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  const std::vector<uint64_t> a = p->pred.layer_activity();
  if (n_layer != a.size()) {
    sfk::set_last_error("sfk_predictor_layer_activity: n_layer does not match the predictor");
    return SFK_ERR_INVALID_ARGUMENT;
  }
  std::copy(a.begin(), a.end(), out);
  return SFK_OK;
}

}  // extern "C"
