"""OffloadManager — the reference's name (packr/offload.py:142-460) for its
GPU <-> pinned-host streaming of W_p and of the 8-bit optimizer state.

Host offload is not part of this build: at B200 memory sizes (180 GB per
GPU) every W_p and the optimizer state stay resident in HBM, and the data-
parallel optimizer shards the state 1/N across GPUs instead.  This class
keeps the reference's public methods so that code written against it runs
unchanged; every tensor stays where it is (ensure / prefetch return at once,
eviction is a no-op).
"""
from __future__ import annotations

import warnings


class OffloadManager:
    def __init__(self, prefetch_depth: int = 1):
        warnings.warn("OffloadManager: host offload is not part of this build; W_p and the optimizer "
                      "state stay resident in HBM", RuntimeWarning, stacklevel=2)
        self.prefetch_depth = prefetch_depth
        self._wp = {}
        self._sequence = []

    def register_wp(self, name, wp_param) -> None:
        self._wp[name] = wp_param

    def set_layer_sequence(self, names) -> None:
        self._sequence = list(names)

    def prefetch_wp(self, name) -> None:
        return None

    def ensure_wp(self, name) -> None:
        return None

    def evict_wp(self, name) -> None:
        return None

    def make_evict_cb(self, name):
        def _cb():
            return None
        return _cb

    @property
    def num_chunks(self) -> int:
        return 0
