"""Whole-model decode step (libkq ``bakan_full_*``), the methods of the
reference's ``FullForwardEngine`` (kandiga/full_forward_engine.py:21-200).

The reference feeds an MLX model's parameters to its Metal engine by name and
then runs ``forward(token_id, position) -> logits``.  Here the same names go
to the CUDA engine (numpy arrays or torch tensors on any device), the model
shape comes from the model config (a dict, or ``packed_dir/config.json``), and
each step replays two CUDA graphs.
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from . import _native as N

DT_F16, DT_BF16, DT_F32, DT_PACKED = 0, 1, 2, 3


def _host(arr, sb: str):
    """-> (contiguous numpy array, ABI dtype code)."""
    try:
        import torch
        if isinstance(arr, torch.Tensor):
            t = arr.detach().contiguous().cpu()
            if t.dtype == torch.bfloat16:
                return t.view(torch.uint16).numpy(), DT_BF16
            if t.dtype == torch.float16:
                return t.numpy(), DT_F16
            if t.dtype == torch.float32:
                return t.numpy(), DT_F32
            if t.dtype == torch.int16:
                return t.numpy().view(np.uint16), DT_BF16 if sb == "bf16" else DT_F16
            arr = t.numpy()
    except ImportError:
        pass
    a = np.ascontiguousarray(arr)
    if a.dtype == np.float16:
        return a, DT_F16
    if a.dtype == np.float32:
        return a, DT_F32
    if a.dtype in (np.uint16, np.int16):  # 16-bit scale/bias/norm bit patterns
        return a.view(np.uint16), DT_BF16 if sb == "bf16" else DT_F16
    if a.dtype in (np.uint32, np.int32, np.uint8):
        return a, DT_PACKED
    raise TypeError(f"unsupported weight dtype {a.dtype}")


class FullForwardEngine:
    """``FullForwardEngine(packed_dir, num_layers, config=None)``;
    ``set_weights(params)``, ``forward(token_id, position)``, ``prefill(ids)``,
    ``reset_cache()``, ``set_kv_cache(...)``, ``set_position(p)``, ``destroy()``."""

    def __init__(self, packed_dir: str, num_layers: int, config: dict | None = None):
        self._lib = N.load()
        if config is None:
            self._engine = self._lib.bakan_full_init(packed_dir.encode(), num_layers)
        else:
            self._engine = self._lib.kq_full_init_json(json.dumps(config).encode(), packed_dir.encode(), num_layers)
        if not self._engine:
            raise RuntimeError("Failed to init full forward engine")
        self.vocab_size = int(self._lib.bakan_full_vocab_size(self._engine))
        self._logits = np.empty(self.vocab_size, dtype=np.float32)

    def set_weight(self, name: str, arr, sb: str = "bf16") -> int:
        a, code = _host(arr, sb)
        shape = (ctypes.c_int64 * a.ndim)(*a.shape)
        return int(self._lib.bakan_full_set_weight(self._engine, name.encode(), a.ctypes.data_as(ctypes.c_void_p),
                                                   a.nbytes, a.ndim, shape, code))

    def set_weights(self, params: dict, sb: str = "bf16"):
        """params: name -> array (MLX parameter names; quantized linears as
        weight / scales / biases).  Builds the engine afterwards."""
        for name, arr in params.items():
            if self.set_weight(name, arr, sb) < 0:
                raise RuntimeError(f"set_weight failed for {name}")
        if self._lib.bakan_full_build(self._engine) != 0:
            raise RuntimeError("Failed to build full forward engine")

    def forward(self, token_id: int, position: int) -> np.ndarray:
        """One decode step; logits float32 [vocab]."""
        vs = ctypes.c_int(0)
        if self._lib.bakan_full_forward(self._engine, int(token_id), int(position),
                                        self._logits.ctypes.data_as(ctypes.c_void_p), ctypes.byref(vs)) != 0:
            raise RuntimeError(f"Forward pass failed at position {position}")
        return self._logits[:vs.value].copy()

    def prefill(self, token_ids) -> np.ndarray:
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        vs = ctypes.c_int(0)
        if self._lib.bakan_full_prefill(self._engine, ids.ctypes.data_as(ctypes.c_void_p), ids.size,
                                        self._logits.ctypes.data_as(ctypes.c_void_p), ctypes.byref(vs)) != 0:
            raise RuntimeError("Prefill failed")
        return self._logits[:vs.value].copy()

    def reset_cache(self):
        self._lib.bakan_full_reset_cache(self._engine)

    def set_kv_cache(self, attn_layer_idx: int, keys: np.ndarray, values: np.ndarray) -> int:
        """keys / values fp16 [num_kv_heads, seq_len, head_dim]."""
        k = np.ascontiguousarray(keys, dtype=np.float16)
        v = np.ascontiguousarray(values, dtype=np.float16)
        return int(self._lib.bakan_full_set_kv_cache(self._engine, attn_layer_idx, k.ctypes.data_as(ctypes.c_void_p),
                                                     v.ctypes.data_as(ctypes.c_void_p), k.shape[1], k.shape[0],
                                                     k.shape[2]))

    def set_linear_state(self, lin_layer_idx: int, state: np.ndarray) -> int:
        """GatedDeltaNet state of the lin_layer_idx-th linear layer, fp32 [v heads, v dim, k dim]."""
        a = np.ascontiguousarray(state, dtype=np.float32)
        return int(self._lib.bakan_full_set_linear_state(self._engine, lin_layer_idx,
                                                         a.ctypes.data_as(ctypes.c_void_p), a.nbytes))

    def set_conv_state(self, lin_layer_idx: int, conv: np.ndarray) -> int:
        """conv1d window of the lin_layer_idx-th linear layer, fp16 [channels, kernel]."""
        a = np.ascontiguousarray(conv, dtype=np.float16)
        return int(self._lib.bakan_full_set_conv_state(self._engine, lin_layer_idx,
                                                       a.ctypes.data_as(ctypes.c_void_p), a.nbytes))

    def set_position(self, position: int) -> int:
        return int(self._lib.bakan_full_set_position(self._engine, position))

    @property
    def position(self) -> int:
        return int(self._lib.kq_full_position(self._engine))

    @property
    def num_layers(self) -> int:
        return int(self._lib.bakan_full_num_layers(self._engine))

    def destroy(self):
        if getattr(self, "_engine", None):
            self._lib.bakan_full_destroy(self._engine)
            self._engine = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass
