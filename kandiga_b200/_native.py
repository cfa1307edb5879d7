"""ctypes binding of libkq.so (include/kq.h).

The library is built in-tree by kandiga_b200/build.py.  There is no fallback:
if the shared object is missing or does not load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB

c_int, c_size_t, c_float, c_void_p = ctypes.c_int, ctypes.c_size_t, ctypes.c_float, ctypes.c_void_p
c_i32p = ctypes.POINTER(ctypes.c_int32)
c_u32p = ctypes.POINTER(ctypes.c_uint32)

KQ_OK = 0
ERRORS = {1: "KQ_ERR_ARG", 2: "KQ_ERR_CUDA", 3: "KQ_ERR_ALLOC", 4: "KQ_ERR_IO", 5: "KQ_ERR_FORMAT",
          6: "KQ_ERR_UNSUPPORTED", 7: "KQ_ERR_WORKSPACE", 8: "KQ_ERR_CAPACITY"}
KQ_ERR_CAPACITY = 8
ERRORS_INV = {v: k for k, v in ERRORS.items()}
DT_F16, DT_BF16, DT_F32 = 0, 1, 2
ACT_SILU, ACT_GELU_TANH = 0, 1
DEV_BAD_EXPERT, DEV_WAIT_TIMEOUT, DEV_BAD_INDEX, DEV_CAPACITY, DEV_RANGE = 1, 2, 4, 8, 16


class KQError(RuntimeError):
    pass


class kq_table_desc(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int32), ("num_experts", ctypes.c_int32),
                ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("bits", ctypes.c_int32),
                ("group_size", ctypes.c_int32), ("sb_dtype", ctypes.c_int32),
                ("activation", ctypes.c_int32)]


class kq_mlx_matrix(ctypes.Structure):
    _fields_ = [("weight", c_void_p), ("scales", c_void_p), ("biases", c_void_p),
                ("weight_stride", ctypes.c_int64), ("sb_stride", ctypes.c_int64)]


# name -> (restype, argtypes)
SIGNATURES = {
    # reference-compatible host ABI
    "bakan_cpu_expert_init": (c_void_p, [ctypes.c_char_p, c_int]),
    "bakan_cpu_expert_mlp": (c_int, [c_void_p, c_int, c_void_p, c_i32p, c_int, c_void_p]),
    "bakan_cpu_expert_mlp_f16": (c_int, [c_void_p, c_int, c_void_p, c_i32p, c_int, c_void_p]),
    "bakan_cpu_expert_mlp_bf16": (c_int, [c_void_p, c_int, c_void_p, c_i32p, c_int, c_void_p]),
    "bakan_cpu_expert_mlp_batch_f16": (c_int, [c_void_p, c_int, c_void_p, c_i32p, c_int, c_int, c_void_p]),
    "bakan_cpu_expert_mlp_prefill_f16": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_i32p,
                                                 c_i32p, c_i32p, c_i32p, c_i32p, c_int, c_void_p]),
    "bakan_cpu_expert_pread_batch": (c_int, [c_void_p, c_int, c_i32p, c_int, c_void_p]),
    "bakan_cpu_expert_destroy": (None, [c_void_p]),
    "bakan_cpu_expert_num_layers": (c_int, [c_void_p]),
    "bakan_forward_init": (c_void_p, [ctypes.c_char_p, c_int]),
    "bakan_forward_set_weight": (c_int, [c_void_p, c_int, c_int, c_void_p, ctypes.c_size_t, c_int, c_int, c_int]),
    "bakan_forward_moe_block": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "bakan_forward_moe_block_normed": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "bakan_forward_destroy": (None, [c_void_p]),
    "bakan_forward_num_layers": (c_int, [c_void_p]),
    "kq_forward_set_params": (c_int, [c_void_p, c_int, ctypes.c_float]),
    "bakan_full_init": (c_void_p, [ctypes.c_char_p, c_int]),
    "bakan_full_set_weight": (c_int, [c_void_p, ctypes.c_char_p, c_void_p, ctypes.c_size_t, c_int,
                                      ctypes.POINTER(ctypes.c_int64), c_int]),
    "bakan_full_build": (c_int, [c_void_p]),
    "bakan_full_forward": (c_int, [c_void_p, c_int, c_int, c_void_p, ctypes.POINTER(c_int)]),
    "bakan_full_prefill": (c_int, [c_void_p, c_void_p, c_int, c_void_p, ctypes.POINTER(c_int)]),
    "bakan_full_reset_cache": (None, [c_void_p]),
    "bakan_full_destroy": (None, [c_void_p]),
    "bakan_full_num_layers": (c_int, [c_void_p]),
    "bakan_full_vocab_size": (c_int, [c_void_p]),
    "bakan_full_set_debug": (None, [c_void_p, c_int]),
    "bakan_full_set_kv_cache": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int]),
    "bakan_full_set_position": (c_int, [c_void_p, c_int]),
    "bakan_full_set_linear_state": (c_int, [c_void_p, c_int, c_void_p, c_int]),
    "bakan_full_set_conv_state": (c_int, [c_void_p, c_int, c_void_p, c_int]),
    "kq_full_init_json": (c_void_p, [ctypes.c_char_p, ctypes.c_char_p, c_int]),
    "kq_full_position": (c_int, [c_void_p]),
    "kq_full_time_steps": (c_int, [c_void_p, c_int, c_int, c_int, ctypes.POINTER(ctypes.c_float)]),
    # device ABI
    "kq_table_create": (c_int, [ctypes.POINTER(kq_table_desc), ctypes.POINTER(c_void_p)]),
    "kq_table_destroy": (c_int, [c_void_p]),
    "kq_table_desc_get": (c_int, [c_void_p, ctypes.POINTER(kq_table_desc)]),
    "kq_table_bytes": (c_size_t, [c_void_p]),
    "kq_table_expert_bytes": (c_size_t, [c_void_p]),
    "kq_table_load_mlx": (c_int, [c_void_p, c_int, c_int, c_int, ctypes.POINTER(kq_mlx_matrix),
                                  ctypes.POINTER(kq_mlx_matrix), ctypes.POINTER(kq_mlx_matrix), c_void_p]),
    "kq_table_load_bkex": (c_int, [c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "kq_table_unpack_mlx": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "kq_moe_workspace_size": (c_size_t, [c_void_p, c_int, c_int]),
    "kq_workspace_init": (c_int, [c_void_p, c_size_t, c_void_p]),
    "kq_router_topk": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "kq_moe_decode": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int,
                              c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "kq_status_read": (c_int, [c_void_p, c_u32p, c_void_p]),
    "kq_moe_prefill_workspace_size": (c_size_t, [c_void_p, c_int, c_int]),
    "kq_moe_prefill": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int,
                               c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "kq_moe_decode_batch_workspace_size": (c_size_t, [c_void_p, c_int]),
    "kq_moe_decode_batch": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                    c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_float,
                                    c_void_p, c_size_t, c_void_p]),
    "kq_moe_decode_static": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                     c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "kq_moe_decode_static_status": (c_int, [c_u32p, c_void_p]),
    "kq_qmat_create": (c_int, [c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "kq_qmat_destroy": (c_int, [c_void_p]),
    "kq_qmat_load_mlx": (c_int, [c_void_p, ctypes.POINTER(kq_mlx_matrix), ctypes.POINTER(kq_mlx_matrix),
                                 c_void_p]),
    "kq_qmat_unpack_mlx": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "kq_gemm_f16_tc": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "kq_dense_gemv": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_float, c_int, c_void_p, c_int,
                              c_void_p]),
    "kq_shared_gate": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int,
                               c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "kq_combine": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p,
                           c_void_p, c_int, c_void_p]),
    "kq_tq3_create": (c_int, [c_int, c_int, c_int, c_void_p, c_size_t, ctypes.POINTER(c_void_p)]),
    "kq_tq3_destroy": (c_int, [c_void_p]),
    "kq_tq3_bytes": (c_size_t, [c_void_p]),
    "kq_tq3_gemv": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p]),
    "kq_tq3_dequant": (c_int, [c_void_p, c_void_p, c_void_p]),
    "kq_tq_create": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_void_p, ctypes.POINTER(c_void_p)]),
    "kq_tq_destroy": (c_int, [c_void_p]),
    "kq_tq_seq_len": (c_int, [c_void_p]),
    "kq_tq_storage_dim": (c_int, [c_void_p]),
    "kq_tq_status": (c_int, [c_void_p, c_u32p, c_void_p]),
    "kq_tq_capacity": (c_int, [c_void_p]),
    "kq_tq_reserve": (c_int, [c_void_p, c_int, c_void_p]),
    "kq_tq_append": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "kq_tq_dequant": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "kq_requantize_mlx": (c_int, [c_void_p, c_void_p, c_void_p, ctypes.c_long, c_int, c_int, c_int, c_int,
                                  c_void_p, c_void_p, c_void_p, c_void_p]),
    "kq_tq_save": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "kq_tq_restore": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_void_p]),
    "kq_tq_export": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "kq_spill_create": (c_int, [ctypes.POINTER(kq_table_desc), c_int, ctypes.POINTER(c_void_p)]),
    "kq_spill_destroy": (c_int, [c_void_p]),
    "kq_spill_pool": (c_void_p, [c_void_p]),
    "kq_spill_host_bytes": (c_size_t, [c_void_p]),
    "kq_spill_store_layer": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p]),
    "kq_spill_fetch": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "kq_spill_prefetch": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p]),
    "kq_spill_stats": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_uint64), c_int, c_void_p]),
    "kq_spill_residency": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "kq_tq_attend_workspace_size": (c_size_t, [c_void_p, c_int]),
    "kq_tq_attend": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    # expert parallelism over peer memory
    "kq_ep_buffer_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "kq_ep_create": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "kq_ep_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "kq_ep_connect": (c_int, [c_void_p, c_void_p]),
    "kq_ep_connect_local": (c_int, [ctypes.POINTER(c_void_p), c_int]),
    "kq_ep_destroy": (None, [c_void_p]),
    "kq_ep_set_wait_ns": (c_int, [c_void_p, ctypes.c_uint64]),
    "kq_ep_dispatch": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int,
                               c_void_p, c_void_p]),
    "kq_ep_receive": (c_int, [c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p),
                              ctypes.POINTER(c_void_p), ctypes.POINTER(c_int), c_void_p]),
    "kq_ep_moe_workspace_size": (c_size_t, [c_void_p, c_void_p]),
    "kq_ep_compute": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "kq_ep_partials": (c_void_p, [c_void_p]),
    "kq_ep_return": (c_int, [c_void_p, c_void_p]),
    "kq_ep_combine": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int,
                              c_void_p]),
    "kq_ep_moe": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p,
                          c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int,
                          c_void_p, c_size_t, c_void_p]),
    "kq_ep_status": (c_int, [c_void_p, c_u32p, c_u32p, c_void_p]),
    "kq_ep_clear_status": (c_int, [c_void_p, c_void_p]),
    "kq_ep_calls": (c_int, [c_void_p, c_u32p]),
}

EP_HANDLE_BYTES = 64
EP_MAX_RANKS = 8

_lib = None


def load(path: str = LIB):
    """Load libkq.so; raises if it is missing (there is no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise KQError(f"libkq.so not found at {path}; build it with `python -m kandiga_b200.build`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str):
    if rc != KQ_OK:
        raise KQError(f"{what} failed: {ERRORS.get(rc, rc)}")
