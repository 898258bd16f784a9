// sfk_tier.h -- host side of the bounded expert tier: the slot pool that
// decides which (layer, expert) bundles occupy the HBM slots, and the
// frequency predictor that picks the next layer's experts to prefetch.
//
// SlotPool restates the reference's tws::SlotPool (src/tws/weight_store.h:
// 69-170 declaration, :173-266 acquire; src/tws/weight_store.cpp:8-147
// capacities and touch): a global LRU, or a layer-stratified pool whose
// per-layer capacities start from a shape-derived split and follow observed
// routing activity, with eviction scoped to the acquiring layer.  The slots
// here are HBM buffers that the expert kernels read in place (the reference
// copies a host slot into a staging tensor right after each acquire), so a
// slot still read by queued kernels is pinned: victims are chosen among the
// unpinned entries only, in the reference's order (own layer's LRU, a free
// slot, the most over-capacity layer).  Without pins the choices are the
// reference's exactly.
//
// ExpertPredictor restates src/predict/predictor.cpp:9-61 (per-layer
// activation counts, most frequent first).  The reference ranks with
// std::partial_sort, which leaves equal counts in an unspecified order; here
// equal counts rank by the lower expert id.
#pragma once
#include <cstdint>
#include <list>
#include <unordered_map>
#include <vector>

namespace sfk {

struct PoolStats {
  uint64_t hits = 0, misses = 0, evictions = 0;
};

class SlotPool {
 public:
  static constexpr uint32_t NONE = 0xFFFFFFFFu;

  // Global LRU over n_slots slots (weight_store.cpp:8-16).
  explicit SlotPool(uint32_t n_slots);
  // Layer-stratified (weight_store.cpp:18-42); n_layer or n_expert 0 gives
  // the global pool.
  SlotPool(uint32_t n_slots, uint32_t n_layer, uint32_t n_expert, uint32_t n_expert_used);

  uint32_t n_slots() const { return n_slots_; }
  bool stratified() const { return stratified_; }
  const PoolStats& stats() const { return stats_; }

  // The slot holding (layer, expert), making it resident on a miss; *miss is
  // set when the caller has to fill the slot.  NONE when the pool has no slot
  // or every candidate victim is pinned.
  uint32_t acquire(uint32_t layer, uint32_t expert, bool* miss);
  bool resident(uint32_t layer, uint32_t expert) const;
  uint32_t slot_of(uint32_t layer, uint32_t expert) const;  // NONE if absent
  // Free slot, or a layer below its capacity with a free slot
  // (weight_store.h:101-123).
  bool has_free_slot() const;
  bool has_free_slot_in_layer(uint32_t layer) const;
  uint32_t layer_capacity(uint32_t layer) const;
  void set_layer_weights(const std::vector<uint64_t>& weights);

  // Pins keep a slot from being chosen as a victim until unpin_all().
  void pin(uint32_t slot);
  void unpin_all();
  uint32_t n_pinned() const { return n_pinned_; }
  // Forget every resident entry (slots become free; statistics are kept).
  void clear();

 private:
  struct Entry {
    uint32_t slot;
    std::list<uint64_t>::iterator it;
  };
  struct LayerState {
    std::list<uint64_t> lru;  // front = most recent
    uint32_t resident = 0;
  };
  static uint64_t key(uint32_t layer, uint32_t expert) { return (uint64_t)layer << 32 | expert; }
  static uint32_t key_layer(uint64_t k) { return (uint32_t)(k >> 32); }
  void recompute_caps(const std::vector<uint64_t>& weights);
  // the least recently used unpinned entry of `lru` (end() if none)
  std::list<uint64_t>::iterator victim(std::list<uint64_t>& lru);
  uint32_t evict(std::list<uint64_t>& lru, std::list<uint64_t>::iterator v);

  uint32_t n_slots_ = 0;
  std::list<uint64_t> lru_;  // global pool
  std::unordered_map<uint64_t, Entry> map_;
  std::vector<uint32_t> free_slots_;
  std::vector<uint8_t> pinned_;
  uint32_t n_pinned_ = 0;
  PoolStats stats_;
  bool stratified_ = false;
  uint32_t n_layer_ = 0, n_expert_ = 0, n_expert_used_ = 0;
  std::vector<LayerState> layers_;
  std::vector<uint32_t> cap_;
};

class ExpertPredictor {
 public:
  ExpertPredictor(uint32_t n_layer, uint32_t n_expert);
  void observe(uint32_t layer, uint32_t expert);
  std::vector<uint32_t> predict(uint32_t layer, uint32_t k);
  double accuracy() const { return predicted_ ? (double)confirmed_ / (double)predicted_ : 0.0; }
  std::vector<uint64_t> layer_activity() const;

 private:
  uint32_t n_layer_, n_expert_;
  std::vector<uint64_t> freq_;  // [layer][expert]
  uint64_t predicted_ = 0, confirmed_ = 0;
  std::vector<uint32_t> last_;
};

}  // namespace sfk
