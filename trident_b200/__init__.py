"""trident_b200: B200-native (sm_100a) implementation of TRIDENT's lossless IVF query path.

Public API (drop-in for the reference's benchmarks/phase4a_suite.py entry points):
    SharedClusterStorage, TridentV4Index (.search / .coarse), load_or_train_clustering,
    choose_tile, merge_shards, save_index / load_index (on-disk artifacts, trident_b200.artifacts),
    and the synthetic dataset generators in trident_b200.datasets.
The search path runs in libtrident_b200.so (C ABI: include/trident_b200.h); see trident_b200.build.
"""
from .artifacts import load_index, save_index
from .clustering import load_or_train_clustering, train_clustering
from .index import SharedClusterStorage, TridentV4Index, choose_tile, merge_shards

__all__ = ["SharedClusterStorage", "TridentV4Index", "choose_tile", "merge_shards", "load_or_train_clustering",
           "train_clustering", "save_index", "load_index"]
