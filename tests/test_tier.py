"""CPU tests of the bounded expert tier's host logic: the slot pool and the
expert predictor through the C ABI.  The scenarios are those of the
reference's own tests (tests/test_slot_pool.cpp, tests/test_predictor.cpp),
plus the pins this build adds because its kernels read the HBM slots in
place."""
import pytest

from strataflow_b200 import build as B
from strataflow_b200.tier import ExpertPredictor, SlotPool


@pytest.fixture(scope="module", autouse=True)
def _lib():
    B.build()


def test_hit_and_miss():  # test_slot_pool.cpp:15-29
    p = SlotPool(2)
    s0, m0 = p.acquire(0, 0)
    s1, m1 = p.acquire(0, 1)
    assert s0 != s1 and m0 and m1
    s2, m2 = p.acquire(0, 0)
    assert s2 == s0 and not m2
    assert p.stats() == {"hits": 1, "misses": 2, "evictions": 0}


def test_slots_handed_out_in_order():  # weight_store.cpp:14 (0, 1, 2, ... first)
    p = SlotPool(3)
    assert [p.acquire(0, e)[0] for e in range(3)] == [0, 1, 2]


def test_lru_eviction():  # test_slot_pool.cpp:31-44
    p = SlotPool(2)
    p.acquire(0, 0)
    p.acquire(0, 1)
    p.acquire(0, 0)          # 0 most recent, 1 least
    p.acquire(0, 2)          # evicts 1
    assert p.resident(0, 0) and p.resident(0, 2) and not p.resident(0, 1)
    assert p.stats()["evictions"] == 1


def test_zero_slots():  # test_slot_pool.cpp:46-50
    p = SlotPool(0)
    assert p.acquire(1, 1) == (None, False)


def _sweep_misses(p, n_layer, k, n_tokens):
    for _ in range(n_tokens):
        for l in range(n_layer):
            for e in range(k):
                p.acquire(l, e)
    return p.stats()["misses"]


def test_stratified_fewer_misses_than_global():  # test_slot_pool.cpp:73-102
    n_layer, n_expert, k, n_tokens = 8, 16, 3, 10
    n_slots = n_layer * k - 1                       # one short of a whole sweep
    g = SlotPool(n_slots)
    s = SlotPool(n_slots, n_layer, n_expert, k)
    assert not g.stratified and s.stratified
    gm = _sweep_misses(g, n_layer, k, n_tokens)
    sm = _sweep_misses(s, n_layer, k, n_tokens)
    assert sm < gm
    assert gm >= n_layer * k * (n_tokens - 1)      # the cyclic pattern thrashes a global LRU
    assert sm < gm // 2 and sm > 0


def test_prior_layer_survives_sweep():  # test_slot_pool.cpp:107-132
    p = SlotPool(12, 4, 8, 2)
    for l in range(4):
        for e in range(2):
            p.acquire(l, e)
    st = p.stats()
    slot, miss = p.acquire(0, 0)
    assert not miss and p.resident(0, 0)
    assert p.stats()["hits"] == st["hits"] + 1 and p.stats()["misses"] == st["misses"]


def test_eviction_scoped_to_layer():  # test_slot_pool.cpp:136-164
    p = SlotPool(12, 4, 8, 2)
    p.acquire(0, 0)
    p.acquire(1, 0)
    p.acquire(3, 0)
    for _ in range(2):
        for e in range(8):
            p.acquire(2, e)
    assert p.resident(0, 0) and p.resident(1, 0) and p.resident(3, 0)
    assert sum(p.resident(2, e) for e in range(8)) <= p.layer_capacity(2)


def test_fully_resident_never_evicts():  # test_slot_pool.cpp:168-190
    p = SlotPool(12, 3, 4, 2)
    assert p.stratified
    for _ in range(2):
        for l in range(3):
            for e in range(4):
                p.acquire(l, e)
    assert p.stats()["evictions"] == 0
    for l in range(3):
        assert p.layer_capacity(l) == 4
        assert all(p.resident(l, e) for e in range(4))


def test_capacity_budget_and_floor():  # test_slot_pool.cpp:195-223
    n_layer, n_expert, k, n_slots = 6, 10, 3, 30
    p = SlotPool(n_slots, n_layer, n_expert, k)

    def check():
        caps = [p.layer_capacity(l) for l in range(n_layer)]
        assert all(k <= c <= n_expert for c in caps) and sum(caps) <= n_slots
    check()
    w = [1] * n_layer
    w[5] = 1000
    p.set_layer_weights(w)
    check()
    assert p.layer_capacity(5) >= p.layer_capacity(0)


def test_capacity_below_topk_still_correct():  # test_slot_pool.cpp:236-298
    n_layer, n_expert, k, n_slots = 8, 16, 4, 20
    p = SlotPool(n_slots, n_layer, n_expert, k)
    caps = [p.layer_capacity(l) for l in range(n_layer)]
    assert all(1 <= c <= n_expert for c in caps) and sum(caps) <= n_slots
    assert any(c < k for c in caps)
    n_tokens = 6
    for _ in range(n_tokens):
        for l in range(n_layer):
            for e in range(k):
                slot, _ = p.acquire(l, e)
                assert slot is not None and p.resident(l, e)
            assert sum(p.resident(l, e) for e in range(n_expert)) <= p.layer_capacity(l)
    s = p.stats()
    assert s["hits"] + s["misses"] == n_tokens * n_layer * k
    assert s["evictions"] <= s["misses"] and s["misses"] > 0 and s["evictions"] > 0


def test_predictor_driven_residency():  # test_slot_pool.cpp:311-400
    n_layer, n_expert, k, n_slots = 4, 8, 2, 9
    pred = ExpertPredictor(n_layer, n_expert)
    p = SlotPool(n_slots, n_layer, n_expert, k)
    cap_hot_before = p.layer_capacity(3)
    for _ in range(50):
        for e in range(n_expert):
            pred.observe(3, e)
        for e in range(n_expert // 2):
            pred.observe(2, e)
        for e in range(k):
            pred.observe(0, e)
            pred.observe(1, e)
    act = pred.layer_activity()
    assert len(act) == n_layer and act[3] > act[2] > act[0]
    p.set_layer_weights(act)
    cap_hot = p.layer_capacity(3)
    assert cap_hot > cap_hot_before
    assert all(cap_hot > p.layer_capacity(l) for l in range(3))
    assert all(p.layer_capacity(l) >= k for l in range(n_layer))
    assert sum(p.layer_capacity(l) for l in range(n_layer)) <= n_slots
    for _ in range(4):
        for e in range(n_expert):
            p.acquire(3, e)
            p.acquire(0, e)
    hot = sum(p.resident(3, e) for e in range(n_expert))
    cold = sum(p.resident(0, e) for e in range(n_expert))
    assert hot >= cold and hot <= cap_hot and cold <= p.layer_capacity(0)


def test_capacity_split_values():
    """The shape-derived split and its refinement, value by value
    (weight_store.cpp:44-119): floor to every layer, spare slots one at a time
    in weight order, stable by index."""
    p = SlotPool(9, 4, 8, 2)
    assert [p.layer_capacity(l) for l in range(4)] == [3, 2, 2, 2]     # the spare slot in index order
    p.set_layer_weights([1, 5, 5, 0])
    assert [p.layer_capacity(l) for l in range(4)] == [2, 3, 2, 2]     # the first of the tied busiest
    p = SlotPool(20, 8, 16, 4)                                           # floor shrinks to 20 // 8 = 2
    assert [p.layer_capacity(l) for l in range(8)] == [3, 3, 3, 3, 2, 2, 2, 2]
    p = SlotPool(100, 3, 4, 2)                                           # never beyond n_expert
    assert [p.layer_capacity(l) for l in range(3)] == [4, 4, 4]


def test_frequency_ranking():  # test_predictor.cpp:8-23
    p = ExpertPredictor(2, 8)
    for _ in range(10):
        p.observe(0, 3)
    for _ in range(5):
        p.observe(0, 5)
    p.observe(0, 1)
    assert p.predict(0, 2) == [3, 5]
    assert len(p.predict(1, 2)) == 2
    assert p.predict(1, 3) == [0, 1, 2]      # equal counts: the lower id first
    assert p.predict(2, 2) == [] and p.predict(0, 0) == []


def test_accuracy_tracking():  # test_predictor.cpp:25-32
    p = ExpertPredictor(1, 4)
    for _ in range(3):
        p.observe(0, 2)
    assert p.predict(0, 1) == [2]
    p.observe(0, 2)
    assert p.accuracy() > 0.0


def test_pinned_slots_are_never_victims():
    """Pinned slots (read by queued kernels) are skipped: the next unpinned
    LRU entry is evicted; with everything pinned there is no slot."""
    p = SlotPool(2)
    a, _ = p.acquire(0, 0)
    b, _ = p.acquire(0, 1)
    p.pin(a)                        # 0 is the LRU entry but pinned
    s, miss = p.acquire(0, 2)
    assert miss and s == b and p.resident(0, 0) and not p.resident(0, 1)
    p.pin(s)
    assert p.acquire(0, 3) == (None, False)
    assert p.stats()["misses"] == 3  # the refused acquire counts nothing
    p.unpin_all()
    s, miss = p.acquire(0, 3)
    assert miss and s == a


def test_pins_in_a_stratified_pool_fall_back_to_free_then_donor():
    """A layer whose own residents are all pinned takes a free slot, then the
    most over-capacity layer's unpinned LRU entry (weight_store.h:221-262)."""
    p = SlotPool(4, 2, 4, 1)                # caps [2, 2]
    s00, _ = p.acquire(0, 0)
    s01, _ = p.acquire(0, 1)
    s10, _ = p.acquire(1, 0)
    p.pin(s00)
    p.pin(s01)
    s02, _ = p.acquire(0, 2)                # layer 0 full and pinned: the free slot
    assert s02 not in (s00, s01, s10) and p.resident(0, 0) and p.resident(0, 1)
    p.pin(s02)
    s03, _ = p.acquire(0, 3)                # no free slot: layer 1's only entry is the donor
    assert s03 == s10 and not p.resident(1, 0)


def test_decode_protocol_keeps_a_steps_experts():
    """The engine's step protocol: unpin at each routing read-back, pin the
    layer's routed experts, prefetch the next layer unpinned.  A prefetch
    never takes a slot the current layer's kernels read, even in a global
    LRU pool the size of one layer's routed set plus one."""
    n_layer, n_expert, k = 4, 8, 2
    p = SlotPool(k + 1)
    pred = ExpertPredictor(n_layer, n_expert)
    import random
    rng = random.Random(5)
    for _ in range(30):
        for l in range(n_layer):
            p.unpin_all()
            ids = rng.sample(range(n_expert), k)
            slots = []
            for x in ids:
                pred.observe(l, x)
                s, _ = p.acquire(l, x)
                assert s is not None
                p.pin(s)
                slots.append(s)
            assert len(set(slots)) == k
            if l + 1 < n_layer:
                for x in pred.predict(l + 1, k):
                    if not p.resident(l + 1, x):
                        s, _ = p.acquire(l + 1, x)
                        assert s is None or s not in slots
            assert all(p.resident(l, x) for x in ids)
