"""ctypes binding of ``libdecode_gemm_b200.so`` (include/decode_gemm_b200.h).

The library is the product; there is no fallback.  ``lib()`` raises when the
shared object is missing or cannot be loaded, so a GPU run without the built
extension fails loudly instead of computing anything elsewhere.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdecode_gemm_b200.so")

ABI_VERSION = 9

LAYOUT_RAW = 0
LAYOUT_PACKED = 1
LAYOUT_PACKED_SWIZZLED = 2
GRID_CLUSTER = -2              # DG_GRID_CLUSTER

FLAG_INJECT_TIMEOUT = 2
FLAG_INDEPENDENT_INPUTS = 4
FLAG_SWAP_AB = 512              # DG_FLAG_SWAP_AB
STATIC_SEM_INTS = 4096          # DG_STATIC_SEM_INTS
STATIC_WS_FLOATS = 2097152      # DG_STATIC_WS_FLOATS

STATUS_OK = 0
ERR_INJECTED_TIMEOUT = 0x51

# Every symbol include/decode_gemm_b200.h declares.
EXPORTED_SYMBOLS = (
    "dg_abi_version", "dg_plan", "dg_make_weight_map", "dg_make_activation_map",
    "dg_launch_with_maps", "dg_launch", "dg_prepack_weight", "dg_padded_n",
    "dg_packed_weight_bytes", "dg_status_string", "dg_flush_l2", "dg_probe_bulk_stream",
    "dg_probe_naive_read", "dg_num_sms", "dg_launch_static_scratch", "dg_probe_mma",
    "dg_launch_gather", "dg_gather_wait", "dg_ipc_export", "dg_ipc_import", "dg_ipc_release",
    "dg_quantize_act", "dg_max_active_clusters", "dg_launch_quantized", "dg_launch_gather_lines",
    "dg_host_device_pointer", "dg_copy_from_host",
)


class DgConfig(ctypes.Structure):
    _fields_ = [
        ("m_tile", ctypes.c_int),
        ("block_n", ctypes.c_int),
        ("subs", ctypes.c_int),
        ("stages", ctypes.c_int),
        ("layout", ctypes.c_int),
        ("pdl", ctypes.c_int),
        ("split_k", ctypes.c_int),
        ("grid_ctas", ctypes.c_int),
        ("epi_warps", ctypes.c_int),
        ("flags", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("pack_rows", ctypes.c_int),
    ]


class DgProblem(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int),
        ("N", ctypes.c_int),
        ("K", ctypes.c_int),
        ("activation", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("weight_scales", ctypes.c_void_p),
        ("activation_scales", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("splitk_ws", ctypes.c_void_p),
        ("splitk_sem", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
    ]


class DgPlanInfo(ctypes.Structure):
    _fields_ = [
        ("grid_x", ctypes.c_uint),
        ("grid_y", ctypes.c_uint),
        ("grid_z", ctypes.c_uint),
        ("block_x", ctypes.c_uint),
        ("smem_bytes", ctypes.c_uint),
        ("num_output_tiles", ctypes.c_int),
        ("padded_n", ctypes.c_int),
        ("stages", ctypes.c_int),
        ("n_mma", ctypes.c_int),
        ("a_rows", ctypes.c_int),
        ("mma_m", ctypes.c_int),
        ("epi_warps", ctypes.c_int),
        ("num_ctas", ctypes.c_int),
        ("max_slabs", ctypes.c_int),
        ("ws_floats", ctypes.c_ulonglong),
        ("sem_ints", ctypes.c_int),
        ("cluster", ctypes.c_int),
        ("error", ctypes.c_char * 96),
    ]


MAX_RANKS = 8                   # DG_MAX_RANKS
ERR_GATHER_WAIT = 0x81


class DgGather(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("ldo", ctypes.c_int),
        ("outputs", ctypes.c_void_p * MAX_RANKS),
        ("flags", ctypes.c_void_p * MAX_RANKS),
        ("sync", ctypes.c_void_p),
    ]


class DgGatherLines(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("ldo", ctypes.c_int),
        ("output", ctypes.c_void_p),
        ("lines", ctypes.c_void_p * MAX_RANKS),
        ("sync", ctypes.c_void_p),
        ("q_out", ctypes.c_void_p),
        ("q_scales", ctypes.c_void_p),
    ]


TensorMap = ctypes.c_uint8 * 128
IpcHandle = ctypes.c_uint8 * 64

_LIB = None


def lib():
    """Load the library (raises if it has not been built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m decode_opt_b200.build` "
            "(there is no non-CUDA implementation of this operator)")
    L = ctypes.CDLL(LIB_PATH)
    cfgp = ctypes.POINTER(DgConfig)
    probp = ctypes.POINTER(DgProblem)
    L.dg_abi_version.restype = ctypes.c_int
    L.dg_plan.argtypes = [cfgp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(DgPlanInfo)]
    L.dg_max_active_clusters.argtypes = [cfgp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.POINTER(ctypes.c_int)]
    L.dg_make_weight_map.argtypes = [cfgp, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    L.dg_make_activation_map.argtypes = [cfgp, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    L.dg_launch_with_maps.argtypes = [cfgp, probp, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_int]
    L.dg_launch_quantized.argtypes = [cfgp, probp, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    L.dg_launch.argtypes = [cfgp, probp, ctypes.c_void_p]
    L.dg_launch_static_scratch.argtypes = [cfgp, probp, ctypes.c_void_p, ctypes.POINTER(DgPlanInfo)]
    L.dg_prepack_weight.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    L.dg_padded_n.argtypes = [ctypes.c_int, ctypes.c_int]
    L.dg_packed_weight_bytes.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.dg_packed_weight_bytes.restype = ctypes.c_ulonglong
    L.dg_status_string.argtypes = [ctypes.c_int]
    L.dg_status_string.restype = ctypes.c_char_p
    L.dg_flush_l2.argtypes = [ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_void_p]
    L.dg_probe_bulk_stream.argtypes = [ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_uint, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    L.dg_probe_naive_read.argtypes = [ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_void_p]
    L.dg_num_sms.restype = ctypes.c_int
    L.dg_launch_gather.argtypes = [cfgp, probp, ctypes.POINTER(DgGather), ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_int]
    L.dg_quantize_act.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    L.dg_launch_gather_lines.argtypes = [cfgp, probp, ctypes.POINTER(DgGatherLines), ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    L.dg_host_device_pointer.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
    L.dg_copy_from_host.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_void_p,
                                    ctypes.c_int]
    L.dg_gather_wait.argtypes = [ctypes.POINTER(DgGather), ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_void_p]
    L.dg_ipc_export.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_ulonglong)]
    L.dg_ipc_import.argtypes = [ctypes.c_void_p, ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_void_p)]
    L.dg_ipc_release.argtypes = [ctypes.c_void_p]
    L.dg_probe_mma.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    if L.dg_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{LIB_PATH}: ABI version {L.dg_abi_version()} != {ABI_VERSION}")
    _LIB = L
    return L
