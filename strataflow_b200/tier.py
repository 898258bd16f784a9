"""Host-side objects of the bounded expert tier (include/sfk.h sfk_pool_*,
sfk_predictor_*): the slot pool and the expert predictor that an engine with
expert_slots below n_layer * n_expert drives every step.

SlotPool mirrors the reference's tws::SlotPool (src/tws/weight_store.h:
69-170): `SlotPool(n_slots)` is the global LRU of the two-argument
constructor, `SlotPool(n_slots, n_layer, n_expert, n_expert_used)` the
layer-stratified pool.  ExpertPredictor mirrors src/predict/predictor.h.
Slot contents live on the device; these objects only keep the bookkeeping.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lib as L


class SlotPool:
    def __init__(self, n_slots: int, n_layer: int = 0, n_expert: int = 0, n_expert_used: int = 0):
        self._lib = L.load()
        h = C.c_void_p()
        L.check(self._lib.sfk_pool_create(n_slots, n_layer, n_expert, n_expert_used, C.byref(h)))
        self.h = h
        self.n_slots = n_slots

    def __del__(self):
        if getattr(self, "h", None):
            self._lib.sfk_pool_free(self.h)
            self.h = None

    def acquire(self, layer: int, expert: int) -> tuple[int | None, bool]:
        """(slot, missed); slot None when no slot could be had."""
        miss = C.c_int32()
        s = self._lib.sfk_pool_acquire(self.h, layer, expert, C.byref(miss))
        return (None if s < 0 else int(s)), bool(miss.value)

    def resident(self, layer: int, expert: int) -> bool:
        return bool(self._lib.sfk_pool_resident(self.h, layer, expert))

    @property
    def stratified(self) -> bool:
        return bool(self._lib.sfk_pool_stratified(self.h))

    def layer_capacity(self, layer: int) -> int:
        return int(self._lib.sfk_pool_layer_capacity(self.h, layer))

    def has_free_slot_in_layer(self, layer: int) -> bool:
        return bool(self._lib.sfk_pool_has_free_slot_in_layer(self.h, layer))

    def set_layer_weights(self, weights) -> None:
        w = np.ascontiguousarray(weights, np.uint64)
        L.check(self._lib.sfk_pool_set_layer_weights(self.h, w.ctypes.data_as(C.c_void_p), len(w)))

    def pin(self, slot: int) -> None:
        L.check(self._lib.sfk_pool_pin(self.h, slot))

    def unpin_all(self) -> None:
        L.check(self._lib.sfk_pool_unpin_all(self.h))

    def stats(self) -> dict:
        out = np.zeros(3, np.uint64)
        L.check(self._lib.sfk_pool_stats(self.h, out.ctypes.data_as(C.c_void_p)))
        return {"hits": int(out[0]), "misses": int(out[1]), "evictions": int(out[2])}


class ExpertPredictor:
    def __init__(self, n_layer: int, n_expert: int):
        self._lib = L.load()
        h = C.c_void_p()
        L.check(self._lib.sfk_predictor_create(n_layer, n_expert, C.byref(h)))
        self.h = h
        self.n_layer, self.n_expert = n_layer, n_expert

    def __del__(self):
        if getattr(self, "h", None):
            self._lib.sfk_predictor_free(self.h)
            self.h = None

    def observe(self, layer: int, expert: int) -> None:
        L.check(self._lib.sfk_predictor_observe(self.h, layer, expert))

    def predict(self, layer: int, k: int) -> list[int]:
        out = np.zeros(max(k, 1), np.uint32)
        n = self._lib.sfk_predictor_predict(self.h, layer, k, out.ctypes.data_as(C.c_void_p))
        return [int(x) for x in out[:n]]

    def accuracy(self) -> float:
        return float(self._lib.sfk_predictor_accuracy(self.h))

    def layer_activity(self) -> list[int]:
        out = np.zeros(self.n_layer, np.uint64)
        L.check(self._lib.sfk_predictor_layer_activity(self.h, out.ctypes.data_as(C.c_void_p), self.n_layer))
        return [int(x) for x in out]
