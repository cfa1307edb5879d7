"""TurboQuant KV cache (PolarQuant 3-bit + 1-bit QJL) on the GPU.

Python mirror of ``TurboQuantCache`` (kandiga/kv_compress.py:22-203): the same
constructor, ``update(keys, values)``, ``keys`` / ``values`` accessors,
``seq_len``, ``memory_bytes``, ``memory_uncompressed`` and
``compression_ratio``, with torch CUDA tensors in place of ``mx.array``.  The
rotation R and the QJL matrix P are drawn exactly as the reference draws them
(kandiga/kv_compress.py:34-44: QR of ``RandomState(seed).randn(D, D)``, then
``choice([-1, 1])`` from the same generator, divided by sqrt(D)).

Storage and compute live in libkq (kq_tq_*): one nibble per element
(3-bit code | sign << 3) plus fp32 scale and zero per vector, preallocated and
grown geometrically instead of concatenated on every append.  ``attend(q)``
adds single-query attention that scores directly on the codes.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _native as N

_DT = {torch.float16: N.DT_F16, torch.bfloat16: N.DT_BF16, torch.float32: N.DT_F32}


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def turboquant_matrices(head_dim: int, seed: int = 42):
    """(R, P) as fp32 numpy arrays, drawn as kandiga/kv_compress.py:34-44."""
    rng = np.random.RandomState(seed)
    random_matrix = rng.randn(head_dim, head_dim).astype(np.float32)
    q, _ = np.linalg.qr(random_matrix)
    qjl = rng.choice([-1.0, 1.0], size=(head_dim, head_dim)).astype(np.float32)
    qjl /= math.sqrt(head_dim)
    return np.ascontiguousarray(q.astype(np.float32)), np.ascontiguousarray(qjl)


class TurboQuantCache:
    """Drop-in compressed KV cache: [batch, heads, seq, head_dim] keys and values."""

    def __init__(self, head_dim: int, num_heads: int, seed: int = 42, capacity: int = 256, device=None):
        if not 1 <= head_dim <= 128:
            raise ValueError("head_dim must be in [1, 128]")
        self.head_dim = head_dim
        self._dstore = 64 if head_dim <= 64 else 128  # storage width of the packed rows
        self.num_heads = num_heads
        self._seed = seed
        self._capacity0 = max(int(capacity), 1)
        self._device = torch.device(device) if device is not None else None
        r, p = turboquant_matrices(head_dim, seed)
        self._r_np, self._p_np = r, p
        dev = self._device if self._device is not None else torch.device("cpu")
        self.rotation = torch.from_numpy(r).to(dev)
        self.rotation_t = self.rotation.t().contiguous()
        self.qjl_proj = torch.from_numpy(p).to(dev)
        self._c = None
        self._batch = None
        self.seq_len = 0

    # ---- storage ---------------------------------------------------------------------------
    def _create(self, batch: int, device):
        self._lib = N.load()
        h = ctypes.c_void_p()
        N.check(self._lib.kq_tq_create(self.head_dim, self.num_heads, batch, self._capacity0,
                                       self._r_np.ctypes.data_as(ctypes.c_void_p),
                                       self._p_np.ctypes.data_as(ctypes.c_void_p), ctypes.byref(h)),
                "kq_tq_create")
        self._c = h
        self._batch = batch
        self._device = device
        self.rotation = self.rotation.to(device)
        self.rotation_t = self.rotation_t.to(device)
        self.qjl_proj = self.qjl_proj.to(device)

    def __del__(self):
        c = getattr(self, "_c", None)
        if c:
            try:
                self._lib.kq_tq_destroy(c)
            except Exception:
                pass
            self._c = None

    def capacity(self) -> int:
        return int(self._lib.kq_tq_capacity(self._c)) if self._c else 0

    def reserve(self, capacity: int):
        N.check(self._lib.kq_tq_reserve(self._c, int(capacity), _stream()), "kq_tq_reserve")

    # ---- reference API -----------------------------------------------------------------------
    def update(self, keys: torch.Tensor, values: torch.Tensor):
        """Compress new entries: keys/values [batch, heads, new_seq, head_dim] on the GPU."""
        if keys.shape != values.shape or keys.dim() != 4:
            raise ValueError("keys and values must both be [batch, heads, seq, head_dim]")
        b, h, t, d = keys.shape
        if h != self.num_heads or d != self.head_dim:
            raise ValueError(f"expected [*, {self.num_heads}, *, {self.head_dim}], got {tuple(keys.shape)}")
        if not keys.is_cuda:
            raise ValueError("TurboQuantCache holds device tensors: pass CUDA tensors")
        if self._c is None:
            self._create(b, keys.device)
        elif b != self._batch:
            raise ValueError(f"batch {b} differs from the cache's batch {self._batch}")
        if t == 0:
            return
        need = self.seq_len + t
        cap = self.capacity()
        if need > cap:
            self.reserve(max(need, 2 * cap))
        dt = keys.dtype if keys.dtype in _DT else torch.float32
        k = keys.to(dt).contiguous()
        v = values.to(dt).contiguous()
        N.check(self._lib.kq_tq_append(self._c, ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()),
                                       _DT[dt], t, _stream()), "kq_tq_append")
        self.seq_len = int(self._lib.kq_tq_seq_len(self._c))

    def _dequant(self, which: int):
        if self._c is None or self.seq_len == 0:
            return None
        out = torch.empty(self._batch, self.num_heads, self.seq_len, self.head_dim, dtype=torch.float16,
                          device=self._device)
        N.check(self._lib.kq_tq_dequant(self._c, which, ctypes.c_void_p(out.data_ptr()), _stream()),
                "kq_tq_dequant")
        return out

    @property
    def keys(self):
        """Decompress and return all keys, fp16 [batch, heads, seq, head_dim] (None if empty)."""
        return self._dequant(0)

    @property
    def values(self):
        """Decompress and return all values (None if empty)."""
        return self._dequant(1)

    @property
    def memory_bytes(self) -> int:
        """Packed size estimate, the reference's formula (kandiga/kv_compress.py:170-188)."""
        if self._c is None or self.seq_len == 0:
            return 0
        n = self._batch * self.num_heads * self.seq_len * self.head_dim
        overhead = self.seq_len * self.num_heads * 4
        return int(n * 0.5 + overhead) * 2

    @property
    def memory_uncompressed(self) -> int:
        if self._c is None or self.seq_len == 0:
            return 0
        return self._batch * self.num_heads * self.seq_len * self.head_dim * 2 * 2

    @property
    def compression_ratio(self) -> float:
        uncomp = self.memory_uncompressed
        if uncomp == 0:
            return 1.0
        return uncomp / self.memory_bytes

    # ---- additions ---------------------------------------------------------------------------
    def export(self, which: int = 0):
        """(codes int8, scales fp32, zeros fp32, signs int8) of keys (0) or values (1) in the
        reference's storage layout: codes/signs [batch, heads, seq, head_dim], scales/zeros
        [batch, heads, seq]."""
        if self._c is None or self.seq_len == 0:
            return None
        shp = (self._batch, self.num_heads, self.seq_len)
        codes = torch.empty(*shp, self.head_dim, dtype=torch.int8, device=self._device)
        signs = torch.empty_like(codes)
        scales = torch.empty(*shp, dtype=torch.float32, device=self._device)
        zeros = torch.empty_like(scales)
        N.check(self._lib.kq_tq_export(self._c, which, ctypes.c_void_p(codes.data_ptr()),
                                       ctypes.c_void_p(signs.data_ptr()), ctypes.c_void_p(scales.data_ptr()),
                                       ctypes.c_void_p(zeros.data_ptr()), _stream()), "kq_tq_export")
        return codes, scales, zeros, signs

    def state(self):
        """The compressed contents: [k_packed, k_scales, k_zeros, v_packed, v_scales, v_zeros]
        (packed uint8 [batch, heads, seq, head_dim/2], two nibbles a byte; scales and zeros
        fp32 [batch, heads, seq]) on the cache's device, or [] when empty."""
        if self._c is None or self.seq_len == 0:
            return []
        shp = (self._batch, self.num_heads, self.seq_len)
        out = []
        for which in (0, 1):
            packed = torch.empty(*shp, self._dstore // 2, dtype=torch.uint8, device=self._device)
            scales = torch.empty(*shp, dtype=torch.float32, device=self._device)
            zeros = torch.empty_like(scales)
            N.check(self._lib.kq_tq_save(self._c, which, ctypes.c_void_p(packed.data_ptr()),
                                         ctypes.c_void_p(scales.data_ptr()), ctypes.c_void_p(zeros.data_ptr()),
                                         _stream()), "kq_tq_save")
            out += [packed, scales, zeros]
        return out

    def load_state(self, state, device=None):
        """Replace the contents with arrays from ``state()`` (torch or numpy, any device)."""
        if len(state) != 6:
            raise ValueError("a TurboQuantCache state holds six arrays")
        kp = torch.as_tensor(state[0])
        if kp.dim() != 4 or kp.shape[1] != self.num_heads or kp.shape[3] != self._dstore // 2:
            raise ValueError(f"packed codes must be [batch, {self.num_heads}, seq, {self._dstore // 2}]")
        b, _, t, _ = kp.shape
        dev = torch.device(device) if device is not None else (self._device or torch.device("cuda"))
        if self._c is None:
            self._create(b, dev)
        elif b != self._batch:
            raise ValueError(f"batch {b} differs from the cache's batch {self._batch}")
        arrs = []
        for i, a in enumerate(state):
            want = torch.uint8 if i % 3 == 0 else torch.float32
            a = torch.as_tensor(a).to(self._device).contiguous()
            if a.dtype != want or a.shape[:3] != (b, self.num_heads, t):
                raise ValueError("state arrays do not match the cache")
            arrs.append(a)
        p = [ctypes.c_void_p(a.data_ptr()) for a in arrs]
        N.check(self._lib.kq_tq_restore(self._c, t, *p, _stream()), "kq_tq_restore")
        self.seq_len = int(self._lib.kq_tq_seq_len(self._c))

    def attend(self, q: torch.Tensor, return_scores: bool = False):
        """softmax(q K^T / sqrt(D)) V over the compressed cache for one query per head.
        q [batch, q_heads, head_dim] (q_heads a multiple of num_heads); returns fp32
        [batch, q_heads, head_dim] (and the scaled logits [batch, q_heads, seq])."""
        if self._c is None or self.seq_len == 0:
            raise ValueError("attention over an empty cache")
        if q.dim() != 3 or q.shape[0] != self._batch or q.shape[2] != self.head_dim:
            raise ValueError("q must be [batch, q_heads, head_dim]")
        hq = q.shape[1]
        dt = q.dtype if q.dtype in _DT else torch.float32
        qc = q.to(dt).contiguous()
        out = torch.empty(self._batch, hq, self.head_dim, dtype=torch.float32, device=self._device)
        scores = (torch.empty(self._batch, hq, self.seq_len, dtype=torch.float32, device=self._device)
                  if return_scores else None)
        ws_bytes = int(self._lib.kq_tq_attend_workspace_size(self._c, hq))
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=self._device)
        N.check(self._lib.kq_tq_attend(self._c, ctypes.c_void_p(qc.data_ptr()), _DT[dt], hq,
                                       ctypes.c_void_p(out.data_ptr()),
                                       ctypes.c_void_p(scores.data_ptr()) if scores is not None else None,
                                       ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream()), "kq_tq_attend")
        return (out, scores) if return_scores else out


# ---- session persistence -----------------------------------------------------------------------

_DTYPE_NAME = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32", torch.uint8: "uint8"}


def save_session(path: str, caches, history=None, tokens_fed: int = 0, model: str = ""):
    """Save per-layer caches in the reference's session layout (kandiga/engine.py:1342-1404):
    ``np.savez_compressed(path, cache_{i}_{j}=...)`` and ``path.replace('.npz', '_meta.json')``
    holding history, tokens_fed, model, dtype_map ({shape, dtype} per array) and layer_info
    ({type, n, offset} per layer).  A layer is a TurboQuantCache (saved compressed: its six
    packed arrays, with head_dim, num_heads and seed in layer_info) or a [keys, values] pair of
    tensors [batch, heads, seq, head_dim] (saved as the reference saves a KVCache: float32 as
    is, 16-bit dtypes as uint16 bit patterns)."""
    import json
    arrays, dtype_map, layer_info = {}, {}, {}
    for i, layer in enumerate(caches):
        if isinstance(layer, TurboQuantCache):
            tensors = layer.state()
            layer_info[str(i)] = {"type": "TurboQuantCache", "n": 6, "offset": layer.seq_len,
                                  "head_dim": layer.head_dim, "num_heads": layer.num_heads, "seed": layer._seed}
        elif layer is not None:
            tensors = list(layer)
            layer_info[str(i)] = {"type": "KVCache", "n": len(tensors),
                                  "offset": int(tensors[0].shape[2]) if tensors else 0}
        else:
            continue
        for j, t in enumerate(tensors):
            t = torch.as_tensor(t).detach().cpu().contiguous()
            key = f"cache_{i}_{j}"
            if t.dtype in (torch.float16, torch.bfloat16):
                arrays[key] = t.view(torch.int16).numpy().view(np.uint16)
            else:
                arrays[key] = t.numpy()
            dtype_map[key] = {"shape": list(t.shape), "dtype": _DTYPE_NAME[t.dtype]}
    np.savez_compressed(path, **arrays)
    with open(path.replace(".npz", "_meta.json"), "w") as f:
        json.dump({"history": list(history or []), "tokens_fed": int(tokens_fed), "model": model,
                   "dtype_map": dtype_map, "layer_info": layer_info}, f)


def load_session(path: str, model: str = None, device="cuda"):
    """Read a session written by save_session: (caches, meta).  TurboQuantCache layers are
    rebuilt on `device` from their packed arrays; other layers come back as lists of tensors
    on `device` with their saved dtypes.  Raises ValueError if `model` is given and differs
    from the saved one (kandiga/engine.py:1421-1422)."""
    import json
    with open(path.replace(".npz", "_meta.json")) as f:
        meta = json.load(f)
    if model is not None and meta["model"] != model:
        raise ValueError(f"Session was for {meta['model']}, not {model}")
    data = np.load(path)
    dtype_map, layer_info = meta.get("dtype_map", {}), meta.get("layer_info", {})
    n_layers = 1 + max((int(k) for k in layer_info), default=-1)
    caches = [None] * n_layers
    for k, info in layer_info.items():
        i = int(k)
        tensors = []
        for j in range(info["n"]):
            key = f"cache_{i}_{j}"
            spec = dtype_map[key]
            a = data[key]
            if spec["dtype"] in ("float16", "bfloat16"):
                t = torch.from_numpy(a.view(np.int16).copy()).view(
                    torch.float16 if spec["dtype"] == "float16" else torch.bfloat16)
            else:
                t = torch.from_numpy(np.ascontiguousarray(a))
            tensors.append(t.reshape(spec["shape"]))
        if info["type"] == "TurboQuantCache":
            c = TurboQuantCache(info["head_dim"], info["num_heads"], seed=info["seed"],
                                capacity=max(info["offset"], 1), device=device)
            if info["offset"] > 0:
                c.load_state(tensors, device=device)
            caches[i] = c
        else:
            caches[i] = [t.to(device) for t in tensors]
    return caches, meta
