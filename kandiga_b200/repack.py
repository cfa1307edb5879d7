"""Expert-file re-quantization on the GPU: the 4-bit -> 3-bit repack of
scripts/repack_experts_3bit.py (parse_header 25-50, repack_layer 169-200,
main 203-243), with the per-projection dequantize / quantize done by
``kq_requantize_mlx`` for all experts of a layer at once on the device.

BKEX container (kandiga/_pack_experts.py:95-132): a 4096-byte header
("BKEX", u32 version = 1, u32 num_experts, u64 expert_size, u32 num_tensors,
then 58-byte descriptors: u8 name_len, char[24] name, u32 offset, u32 nbytes,
u32 d0, u32 d1, u8 dtype (0 uint32, 1 bf16)) followed by num_experts blobs of
expert_size bytes.  The repacked file keeps the reference's tensor order
(gate, up, down projection; weight, scales, biases) with 3-bit weights stored
as uint32 [rows, cols * 3 / 32] and bf16 scales and biases [rows, cols / 64].
"""
from __future__ import annotations

import ctypes
import os
import struct

import numpy as np
import torch

from . import _native as N

HEADER_SIZE = 4096
GROUP_SIZE = 64
PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def parse_header(hdr: bytes):
    """(num_experts, expert_size, [{name, offset, nbytes, shape, dtype}])."""
    if hdr[:4] != b"BKEX":
        raise ValueError("not a BKEX layer file")
    num_experts, = struct.unpack_from("<I", hdr, 8)
    expert_size, = struct.unpack_from("<Q", hdr, 12)
    n, = struct.unpack_from("<I", hdr, 20)
    tensors, pos = [], 24
    for _ in range(n):
        ln = hdr[pos]
        name = hdr[pos + 1:pos + 1 + ln].decode("ascii")
        off, nb, d0, d1 = struct.unpack_from("<IIII", hdr, pos + 25)
        tensors.append({"name": name, "offset": off, "nbytes": nb, "shape": (d0, d1),
                        "dtype": "uint32" if hdr[pos + 41] == 0 else "bfloat16"})
        pos += 42
    return num_experts, expert_size, tensors


def build_header(num_experts: int, expert_size: int, tensors) -> bytes:
    buf = bytearray(HEADER_SIZE)
    buf[0:4] = b"BKEX"
    struct.pack_into("<IIQI", buf, 4, 1, num_experts, expert_size, len(tensors))
    pos = 24
    for t in tensors:
        name = t["name"].encode("ascii")
        buf[pos] = len(name)
        buf[pos + 1:pos + 1 + len(name)] = name
        struct.pack_into("<IIIIB", buf, pos + 25, t["offset"], t["nbytes"], t["shape"][0], t["shape"][1],
                         0 if t["dtype"] == "uint32" else 1)
        pos += 42
    return bytes(buf)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def requantize(weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, cols: int, src_bits: int,
               dst_bits: int, sb_dtype: str = "bf16"):
    """One MLX-layout matrix (device tensors: packed weight bytes or words, 16-bit scales and
    biases) dequantized and quantized again at dst_bits: (packed uint8, scales int16, biases int16)."""
    rows = scales.shape[0]
    w_out = torch.empty(rows, cols * dst_bits // 8, dtype=torch.uint8, device=weight.device)
    s_out = torch.empty(rows, cols // GROUP_SIZE, dtype=torch.int16, device=weight.device)
    b_out = torch.empty_like(s_out)
    lib = N.load()
    N.check(lib.kq_requantize_mlx(ctypes.c_void_p(weight.data_ptr()), ctypes.c_void_p(scales.data_ptr()),
                                  ctypes.c_void_p(biases.data_ptr()), rows, cols, src_bits, dst_bits,
                                  N.DT_BF16 if sb_dtype == "bf16" else N.DT_F16,
                                  ctypes.c_void_p(w_out.data_ptr()), ctypes.c_void_p(s_out.data_ptr()),
                                  ctypes.c_void_p(b_out.data_ptr()), _stream()), "kq_requantize_mlx")
    return w_out, s_out, b_out


def repack_layer(input_path: str, output_path: str, bits: int = 3, device="cuda") -> int:
    """Re-quantize every expert of one BKEX layer file to `bits`; returns the new expert size."""
    with open(input_path, "rb") as f:
        data = f.read()
    num_experts, esz, descs = parse_header(data[:HEADER_SIZE])
    by_name = {d["name"]: d for d in descs}
    payload = torch.frombuffer(bytearray(data[HEADER_SIZE:HEADER_SIZE + num_experts * esz]),
                               dtype=torch.uint8).to(device).view(num_experts, esz)
    parts, layout, off = [], [], 0
    for proj in PROJECTIONS:
        w, s, b = (by_name[f"{proj}.{k}"] for k in ("weight", "scales", "biases"))
        rows, groups = s["shape"]
        cols = groups * GROUP_SIZE
        src_bits = w["shape"][1] * 32 // cols
        if w["dtype"] != "uint32" or src_bits not in (3, 4) or s["dtype"] != "bfloat16":
            raise ValueError(f"{input_path}: {proj} is not a 3/4-bit matrix with bf16 scales")
        ws = payload[:, w["offset"]:w["offset"] + w["nbytes"]].contiguous()
        ss = payload[:, s["offset"]:s["offset"] + s["nbytes"]].contiguous().view(torch.int16)
        bs = payload[:, b["offset"]:b["offset"] + b["nbytes"]].contiguous().view(torch.int16)
        # all experts' rows at once: [E * rows] rows of the same width
        wq, sq, bq = requantize(ws.view(num_experts * rows, -1), ss.view(num_experts * rows, -1),
                                bs.view(num_experts * rows, -1), cols, src_bits, bits, "bf16")
        for name, t, shape, dt in ((f"{proj}.weight", wq, (rows, cols * bits // 32), "uint32"),
                                   (f"{proj}.scales", sq, (rows, groups), "bfloat16"),
                                   (f"{proj}.biases", bq, (rows, groups), "bfloat16")):
            t = t.view(torch.uint8).reshape(num_experts, -1)
            layout.append({"name": name, "offset": off, "nbytes": t.shape[1], "shape": shape, "dtype": dt})
            parts.append(t)
            off += t.shape[1]
    out = torch.cat(parts, dim=1).cpu().numpy()
    with open(output_path, "wb") as f:
        f.write(build_header(num_experts, off, layout))
        f.write(out.tobytes())
    if os.path.getsize(output_path) != HEADER_SIZE + num_experts * off:
        raise RuntimeError(f"{output_path}: size mismatch")
    return off


def repack_dir(packed_dir: str, output_dir: str = None, bits: int = 3, device="cuda"):
    """Repack every layer_XX.bin of packed_dir into output_dir (default: packed_3bit beside it)."""
    if output_dir is None:
        output_dir = os.path.join(os.path.dirname(os.path.abspath(packed_dir)), f"packed_{bits}bit")
    os.makedirs(output_dir, exist_ok=True)
    files = sorted(f for f in os.listdir(packed_dir) if f.startswith("layer_") and f.endswith(".bin"))
    sizes = [repack_layer(os.path.join(packed_dir, f), os.path.join(output_dir, f), bits, device) for f in files]
    return output_dir, sizes
