"""ctypes binding of libtrident_b200.so (the C ABI in include/trident_b200.h).

The library is built in-tree by trident_b200/build.py. There is no fallback: if the shared object
is missing or cannot be loaded, importing the search path raises, on purpose.
"""
import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libtrident_b200.so")

TRIDENT_OK = 0
TRIDENT_ERR_INVALID = 1
TRIDENT_ERR_WORKSPACE = 2
TRIDENT_ERR_CUDA = 3
TRIDENT_ERR_UNSUPPORTED = 4

MODE_AUTO = -1
MODE_CASCADE = 2
MODE_CM_FP32 = 10

STATS_LEN = 8
STAT_NAMES = ("candidates", "scanned_dims", "survivors", "inserted", "coarse_recheck", "items", "r6", "r7")

EXPORTED = (
    "trident_version", "trident_last_error", "trident_index_check", "trident_workspace_size", "trident_p_init",
    "trident_route", "trident_search", "trident_search_profiled", "trident_launch_count", "trident_coarse",
    "trident_merge_shards", "trident_search_noalloc", "trident_search_prep", "trident_search_seed",
    "trident_search_finish", "trident_workspace_status", "trident_set_wait_limits",
    "trident_noalloc_workspace_bytes", "trident_assign", "trident_stage_y_tensor",
)
QINFO_LEN = 4
PHASES = ("coarse", "pairs", "seed", "scan", "merge")

# device-side status word of a workspace (trident_workspace_status)
INDEX_TENSOR_STAGE_Y_ALWAYS = 1
STATUS_OK = 0
STATUS_LOCK_TIMEOUT = 1
STATUS_MMA_TIMEOUT = 2


def noalloc_workspace_bytes() -> int:
    """Size of the fixed workspace behind trident_search_noalloc, as compiled into the library."""
    return int(lib().trident_noalloc_workspace_bytes())


class TridentError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"trident error {code}: {msg}")
        self.code = code


class TridentIndexDesc(ctypes.Structure):
    """Mirror of `trident_index` (include/trident_b200.h)."""
    _fields_ = [
        ("N", ctypes.c_int64),
        ("D", ctypes.c_int32),
        ("D_pad", ctypes.c_int32),
        ("nlist", ctypes.c_int32),
        ("tile_size", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("xb_sorted", ctypes.c_void_p),
        ("orig_ids_sorted", ctypes.c_void_p),
        ("list_row_off", ctypes.c_void_p),
        ("list_tile_off", ctypes.c_void_p),
        ("codes", ctypes.c_void_p),
        ("vmin", ctypes.c_void_p),
        ("delta", ctypes.c_void_p),
        ("eps", ctypes.c_void_p),
        ("centroids", ctypes.c_void_p),
        ("centroid_norm_sq", ctypes.c_void_p),
        ("pca_mean", ctypes.c_void_p),
        ("pca_rot", ctypes.c_void_p),
        ("centroid_norm_max", ctypes.c_float),
        ("lb_rel_slack", ctypes.c_float),
        ("row_p", ctypes.c_void_p),
    ]


_LIB = None


def lib():
    """Load the CUDA library (once). Raises ImportError when it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m trident_b200.build` "
                          "(or __graft_entry__.build()); there is no CPU fallback")
    L = ctypes.CDLL(LIB_PATH)
    P, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    DP = ctypes.POINTER(TridentIndexDesc)
    L.trident_version.restype = ctypes.c_int
    L.trident_last_error.restype = ctypes.c_char_p
    L.trident_index_check.argtypes = [DP]
    L.trident_workspace_size.argtypes = [DP, i32, i32, i32, ctypes.POINTER(sz)]
    L.trident_p_init.argtypes = [i32, i32, i32, i32]
    L.trident_p_init.restype = i32
    L.trident_route.argtypes = [DP, i32, i32, ctypes.c_double]
    L.trident_route.restype = i32
    L.trident_stage_y_tensor.argtypes = [DP, i32, i32, i32, i32]
    L.trident_stage_y_tensor.restype = i32
    L.trident_search.argtypes = [DP, P, i32, i32, i32, i32, i32, P, sz, P, P, P, P]
    L.trident_search_profiled.argtypes = [DP, P, i32, i32, i32, i32, i32, P, sz, P, P, P, P, P]
    L.trident_launch_count.restype = i64
    L.trident_coarse.argtypes = [DP, P, i32, i32, P, sz, P, P, P, P, P]
    L.trident_merge_shards.argtypes = [P, P, i32, i32, i32, P, P, P]
    L.trident_search_noalloc.argtypes = [DP, P, i32, i32, i32, i32, i32, P, P, P, P]
    L.trident_search_prep.argtypes = [DP, P, i32, i32, P, sz, P, P, P, P]
    L.trident_search_seed.argtypes = [DP, P, i32, i32, i32, i32, i32, P, P, P, P, sz, P, P, P]
    L.trident_search_finish.argtypes = [DP, P, i32, i32, i32, i32, i32, P, P, sz, P, P, P, P]
    L.trident_workspace_status.argtypes = [P, P, ctypes.POINTER(i32)]
    L.trident_set_wait_limits.argtypes = [i64, i64]
    L.trident_noalloc_workspace_bytes.restype = sz
    L.trident_assign.argtypes = [P, i64, i32, P, P, i32, P, P, P]
    for name in ("trident_index_check", "trident_workspace_size", "trident_search", "trident_search_profiled",
                 "trident_coarse", "trident_merge_shards", "trident_search_noalloc", "trident_search_prep",
                 "trident_search_seed", "trident_search_finish", "trident_workspace_status",
                 "trident_set_wait_limits", "trident_assign"):
        getattr(L, name).restype = ctypes.c_int
    _LIB = L
    return L


def check(rc: int) -> None:
    if rc != TRIDENT_OK:
        raise TridentError(rc, lib().trident_last_error().decode(errors="replace"))


def set_wait_limits(lock_spins: int = -1, mma_polls: int = -1) -> None:
    """Process-wide limits of the kernels' bounded waits (-1: the defaults)."""
    check(lib().trident_set_wait_limits(int(lock_spins), int(mma_polls)))


def last_error() -> str:
    return lib().trident_last_error().decode(errors="replace")
