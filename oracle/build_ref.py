"""Build the reference's own scalar expert-MLP C into oracle/_ref/ (test infrastructure).

The reference's native expert code lives in Objective-C files
(kandiga/metal/kandiga_cpu_expert.m, kandiga/metal/kandiga_cpu_expert_lg.m) that
need Foundation and Grand Central Dispatch, so the files as a whole cannot be
compiled with gcc on x86_64.  The arithmetic functions inside them are plain C,
and on x86_64 their NEON branches are compiled out, leaving the scalar `#else`
branches.  This recipe extracts exactly those functions by name from the files
where they lie, pipes them to gcc on stdin together with a small driver written
here, and writes only the resulting shared objects into oracle/_ref/.  No
reference source is written into this repository.

Functions taken from kandiga/metal/kandiga_cpu_expert.m:
    bf16_to_float, float_to_half, half_to_float, cpu_dequant_matvec_3bit,
    cpu_dequant_matvec_4bit, compute_single_expert, compute_single_expert_3bit
    and the model constants (#define lines 37-65).
Functions taken from kandiga/metal/kandiga_cpu_expert_lg.m:
    the Engine struct, bf16_to_f32, matvec3, matvec4, expert_mlp.

Usage: python oracle/build_ref.py [reference_root]
Outputs: oracle/_ref/libref_expert.so, oracle/_ref/libref_expert_lg.so
"""
from __future__ import annotations

import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
def reference_root():
    """The kandiga project tree: $KQ_REFERENCE_ROOT, else a directory named
    `reference` beside this repository's root; None when neither exists."""
    env = os.environ.get("KQ_REFERENCE_ROOT")
    if env:
        return env if os.path.isdir(env) else None
    beside = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return beside if os.path.isdir(beside) else None


DEFAULT_REF = reference_root()

CFLAGS = ["-O2", "-ffp-contract=off", "-fPIC", "-shared", "-fopenmp", "-std=gnu11", "-w"]


def _extract_function(src: str, name: str) -> str:
    """Return the full definition of C function `name` (signature through its closing brace)."""
    m = re.search(r"^static[^\n;{]*\b" + re.escape(name) + r"\s*\(", src, re.M)
    if not m:
        raise RuntimeError(f"function {name} not found")
    start = m.start()
    brace = src.index("{", m.end())
    depth = 0
    i = brace
    while i < len(src):
        c = src[i]
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return src[start:i + 1] + "\n"
        i += 1
    raise RuntimeError(f"unbalanced braces in {name}")


def _extract_defines(src: str, names: list[str]) -> str:
    out = []
    for line in src.splitlines():
        m = re.match(r"#define\s+(\w+)\s", line)
        if m and m.group(1) in names:
            out.append(line)
    return "\n".join(out) + "\n"


def _extract_struct(src: str, tag: str) -> str:
    m = re.search(r"typedef struct \{.*?\}\s*" + re.escape(tag) + r";", src, re.S)
    if not m:
        raise RuntimeError(f"struct {tag} not found")
    return m.group(0) + "\n"


PRELUDE = """
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
"""

# Driver for the small variant (written here): exported entry points that call
# the reference's static functions, with OpenMP standing in for the GCD fan-out
# of kandiga/metal/kandiga_cpu_expert.m:522-543.
DRIVER_SMALL = r"""
int ref_expert_size(int bits) { return bits == 3 ? (int)EXPERT_SIZE_3BIT : (int)EXPERT_SIZE; }
int ref_hidden(void) { return HIDDEN_SIZE; }
int ref_inter(void) { return EXPERT_DIM; }
void ref_matvec3(const uint8_t* w, const uint16_t* s, const uint16_t* b, const float* x,
                 float* out, int od, int id) {
    cpu_dequant_matvec_3bit(w, s, b, x, out, od, id, GROUP_SIZE);
}
void ref_matvec4(const uint32_t* w, const uint16_t* s, const uint16_t* b, const float* x,
                 float* out, int od, int id) {
    cpu_dequant_matvec_4bit(w, s, b, x, out, od, id, GROUP_SIZE);
}
int ref_expert(int bits, const char* blob, const float* x, float* out) {
    return bits == 3 ? compute_single_expert_3bit(blob, x, out) : compute_single_expert(blob, x, out);
}
/* layer: num_experts * expert_size bytes (BKEX payload, header stripped).
 * x [T][HIDDEN_SIZE], idx [T][K], out [T][K][HIDDEN_SIZE]. */
int ref_moe_layer(int bits, const char* layer, const float* x, const int32_t* idx,
                  int T, int K, float* out, int threads) {
    long esz = bits == 3 ? (long)EXPERT_SIZE_3BIT : (long)EXPERT_SIZE;
    long total = (long)T * K;
    int err = 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1) reduction(|:err)
    for (long tk = 0; tk < total; tk++) {
        const char* blob = layer + (long)idx[tk] * esz;
        const float* xt = x + (tk / K) * HIDDEN_SIZE;
        err |= ref_expert(bits, blob, xt, out + tk * HIDDEN_SIZE);
    }
    return err;
}
"""

# Driver for the large (dimension-from-header) variant.
DRIVER_LG = r"""
int ref_lg_expert(int bits, int use_gelu, int hidden, int inter, const size_t* offs,
                  const char* data, const float* x, float* out) {
    Engine e;
    memset(&e, 0, sizeof(e));
    e.hidden_size = hidden; e.expert_dim = inter; e.bits = bits; e.use_gelu = use_gelu;
    e.gate_w_off = offs[0]; e.gate_s_off = offs[1]; e.gate_b_off = offs[2];
    e.up_w_off = offs[3];   e.up_s_off = offs[4];   e.up_b_off = offs[5];
    e.down_w_off = offs[6]; e.down_s_off = offs[7]; e.down_b_off = offs[8];
    float* scratch = (float*)malloc(sizeof(float) * 3 * (size_t)inter);
    int r = expert_mlp(&e, data, x, out, scratch);
    free(scratch);
    return r;
}
"""


def build(ref_root: str | None = None) -> list[str]:
    ref_root = ref_root or DEFAULT_REF
    if ref_root is None:
        raise FileNotFoundError("reference tree not found: set KQ_REFERENCE_ROOT")
    small_path = os.path.join(ref_root, "kandiga", "metal", "kandiga_cpu_expert.m")
    lg_path = os.path.join(ref_root, "kandiga", "metal", "kandiga_cpu_expert_lg.m")
    if not (os.path.exists(small_path) and os.path.exists(lg_path)):
        raise FileNotFoundError(f"reference sources not found under {ref_root}")
    os.makedirs(OUT, exist_ok=True)
    built = []

    small = open(small_path).read()
    defines = _extract_defines(small, [
        "MAX_EXPERTS", "HIDDEN_SIZE", "EXPERT_DIM", "GROUP_SIZE", "HEADER_SIZE", "EXPERT_SIZE",
        "GATE_WEIGHT_OFF", "GATE_SCALES_OFF", "GATE_BIASES_OFF", "UP_WEIGHT_OFF", "UP_SCALES_OFF",
        "UP_BIASES_OFF", "DOWN_WEIGHT_OFF", "DOWN_SCALES_OFF", "DOWN_BIASES_OFF",
        "GATE_WEIGHT_OFF_3", "GATE_SCALES_OFF_3", "GATE_BIASES_OFF_3", "UP_WEIGHT_OFF_3",
        "UP_SCALES_OFF_3", "UP_BIASES_OFF_3", "DOWN_WEIGHT_OFF_3", "DOWN_SCALES_OFF_3",
        "DOWN_BIASES_OFF_3", "EXPERT_SIZE_3BIT"])
    funcs = "".join(_extract_function(small, n) for n in [
        "bf16_to_float", "float_to_half", "half_to_float", "cpu_dequant_matvec_3bit",
        "cpu_dequant_matvec_4bit", "compute_single_expert", "compute_single_expert_3bit"])
    out_small = os.path.join(OUT, "libref_expert.so")
    subprocess.run(["gcc", *CFLAGS, "-x", "c", "-", "-o", out_small, "-lm"],
                   input=(PRELUDE + defines + funcs + DRIVER_SMALL).encode(), check=True)
    built.append(out_small)

    lg = open(lg_path).read()
    defines_lg = _extract_defines(lg, ["MAX_EXPERTS", "HEADER_SIZE", "GROUP_SIZE"])
    struct = _extract_struct(lg, "Engine")
    funcs_lg = "".join(_extract_function(lg, n) for n in [
        "bf16_to_f32", "matvec3", "matvec4", "expert_mlp"])
    out_lg = os.path.join(OUT, "libref_expert_lg.so")
    subprocess.run(["gcc", *CFLAGS, "-x", "c", "-", "-o", out_lg, "-lm"],
                   input=(PRELUDE + defines_lg + struct + funcs_lg + DRIVER_LG).encode(), check=True)
    built.append(out_lg)
    return built


if __name__ == "__main__":
    for p in build(sys.argv[1] if len(sys.argv) > 1 else None):
        print(p)
