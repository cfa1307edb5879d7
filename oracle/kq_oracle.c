/*
 * kq_oracle.c -- CPU restatement of the reference's quantized routed-expert path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load this library, and only as
 * the checker.  The product path (kandiga_b200/) never calls it.
 *
 * Every function restates, in this file's own code, the arithmetic of a
 * reference function (paths relative to the kandiga project root):
 *
 *   kqo_code3 / kqo_unpack3   3-bit MLX packing, 8 codes per 3 bytes, LSB-first:
 *                             kandiga/metal/kandiga_cpu_expert.m:194-201
 *   kqo_unpack4               4-bit nibbles in uint32, LSB-first:
 *                             kandiga/metal/kandiga_cpu_expert.m:285-291
 *   kqo_matvec                affine group dequant + fp32 dot, accumulated in the
 *                             scalar branch's order (group, pack, code):
 *                             kandiga/metal/kandiga_cpu_expert.m:182-214 (3-bit),
 *                             :280-296 (4-bit); kandiga_cpu_expert_lg.m:159-168,209-214
 *   kqo_expert_mlp            gate, up, silu(g)*u with expf (or GELU-tanh), down:
 *                             kandiga/metal/kandiga_cpu_expert.m:355-401,
 *                             kandiga/metal/kandiga_cpu_expert_lg.m:220-268
 *   kqo_router_topk           softmax + K rounds of strict-greater argmax
 *                             (lowest index wins ties) + renormalisation:
 *                             kandiga/metal/moe_block.metal:419-505
 *   kqo_combine               out = [res] + sum_k w_k y_k [+ gate*shared]:
 *                             kandiga/metal/moe_block.metal:515-584
 *
 * Pinning: tests compare this file bit-for-bit against the reference's own
 * scalar C compiled from the reference tree by oracle/build_ref.py (the router
 * and combine are Metal-only in the reference: parity unpinned for those two).
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared -fopenmp (oracle/build.py).
 * fp-contract is off so the accumulation order and rounding match the
 * reference's scalar C built the same way.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>

/* ---- 16-bit float helpers ------------------------------------------------ */
static inline float kqo_from_bf16(uint16_t v) {
    uint32_t b = (uint32_t)v << 16; float f; memcpy(&f, &b, 4); return f;
}
static inline float kqo_from_f16(uint16_t v) {
    _Float16 h; memcpy(&h, &v, 2); return (float)h;
}
static inline uint16_t kqo_to_f16(float f) {
    _Float16 h = (_Float16)f; uint16_t r; memcpy(&r, &h, 2); return r;
}
/* sb_dtype: 0 = bf16 (reference BKEX files), 1 = fp16 (synthetic configs) */
static inline float kqo_sb(uint16_t v, int sb_dtype) {
    return sb_dtype ? kqo_from_f16(v) : kqo_from_bf16(v);
}

/* ---- unpack ---------------------------------------------------------------- */
/* j-th 3-bit code of a packed row: bits [3j, 3j+3) of the little-endian byte
 * stream.  Pack p = j/8 occupies bytes 3p..3p+2. */
int kqo_code3(const uint8_t* row, int j) {
    const uint8_t* b = row + 3 * (j >> 3);
    uint32_t word = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16);
    return (int)((word >> (3 * (j & 7))) & 7u);
}

void kqo_unpack3(const uint8_t* row, int n, uint8_t* codes) {
    for (int j = 0; j < n; j++) codes[j] = (uint8_t)kqo_code3(row, j);
}

void kqo_unpack4(const uint32_t* row, int n, uint8_t* codes) {
    for (int j = 0; j < n; j++) codes[j] = (uint8_t)((row[j >> 3] >> (4 * (j & 7))) & 0xFu);
}

/* Pack codes back into the MLX byte layout (inverse of the unpack above). */
void kqo_pack3(const uint8_t* codes, int n, uint8_t* row) {
    memset(row, 0, (size_t)n * 3 / 8);
    for (int j = 0; j < n; j++) {
        int bit = 3 * j;
        uint32_t v = (uint32_t)(codes[j] & 7u) << (bit & 7);
        row[bit >> 3] |= (uint8_t)(v & 0xFFu);
        if ((bit & 7) > 5) row[(bit >> 3) + 1] |= (uint8_t)(v >> 8);
    }
}

void kqo_pack4(const uint8_t* codes, int n, uint32_t* row) {
    memset(row, 0, (size_t)n / 2);
    for (int j = 0; j < n; j++) row[j >> 3] |= (uint32_t)(codes[j] & 0xFu) << (4 * (j & 7));
}

/* ---- affine group dequant + matvec ---------------------------------------- */
/* out[r] = sum_g sum_i (q * s_g + b_g) * x_i, fp32, accumulated in the order
 * group -> pack of 8 -> code, exactly as the reference's scalar branch.
 * variant 0: every product is added to the accumulator in turn
 *            (kandiga/metal/kandiga_cpu_expert.m:203-210, :289-293 and
 *            kandiga/metal/kandiga_cpu_expert_lg.m:213).
 * variant 1: 3-bit only, the 8 products of a pack are summed left to right
 *            and that sum is added (kandiga/metal/kandiga_cpu_expert_lg.m:163-167). */
void kqo_matvec_v(int bits, int variant, const void* weight, const uint16_t* scales,
                  const uint16_t* biases, int sb_dtype, const float* x, float* out, int out_dim,
                  int in_dim, int gs) {
    int ngroups = in_dim / gs;
    for (int r = 0; r < out_dim; r++) {
        const uint16_t* s_row = scales + (size_t)r * ngroups;
        const uint16_t* b_row = biases + (size_t)r * ngroups;
        float acc = 0.0f;
        if (bits == 3) {
            const uint8_t* w_row = (const uint8_t*)weight + (size_t)r * (in_dim * 3 / 8);
            for (int g = 0; g < ngroups; g++) {
                float s = kqo_sb(s_row[g], sb_dtype), b = kqo_sb(b_row[g], sb_dtype);
                for (int p = 0; p < gs / 8; p++) {
                    int base = g * gs + p * 8;
                    if (variant == 1) {
                        float ps = ((float)kqo_code3(w_row, base) * s + b) * x[base];
                        for (int t = 1; t < 8; t++)
                            ps = ps + ((float)kqo_code3(w_row, base + t) * s + b) * x[base + t];
                        acc += ps;
                    } else {
                        for (int t = 0; t < 8; t++) {
                            float v = (float)kqo_code3(w_row, base + t);
                            acc += (v * s + b) * x[base + t];
                        }
                    }
                }
            }
        } else {
            const uint32_t* w_row = (const uint32_t*)weight + (size_t)r * (in_dim / 8);
            for (int g = 0; g < ngroups; g++) {
                float s = kqo_sb(s_row[g], sb_dtype), b = kqo_sb(b_row[g], sb_dtype);
                for (int p = 0; p < gs / 8; p++) {
                    uint32_t word = w_row[g * (gs / 8) + p];
                    int base = g * gs + p * 8;
                    for (int t = 0; t < 8; t++) {
                        float v = (float)((word >> (4 * t)) & 0xFu);
                        acc += (v * s + b) * x[base + t];
                    }
                }
            }
        }
        out[r] = acc;
    }
}

void kqo_matvec(int bits, const void* weight, const uint16_t* scales, const uint16_t* biases,
                int sb_dtype, const float* x, float* out, int out_dim, int in_dim, int gs) {
    kqo_matvec_v(bits, 0, weight, scales, biases, sb_dtype, x, out, out_dim, in_dim, gs);
}

/* ---- one expert ------------------------------------------------------------ */
/* An expert is nine tensors: gate/up/down x {weight, scales, biases}.  The
 * caller passes their pointers (the reference reads them from one BKEX blob at
 * fixed offsets; kandiga/metal/kandiga_cpu_expert.m:44-65). */
typedef struct {
    const void* w[3];         /* gate, up, down packed weights */
    const uint16_t* s[3];     /* scales */
    const uint16_t* b[3];     /* biases */
} kqo_expert;

/* act: 0 = SwiGLU (silu(g) = g / (1 + expf(-g))), 1 = GELU-tanh gate.
 * variant: accumulation order of kqo_matvec_v (0 small library, 1 large). */
void kqo_expert_mlp(int bits, int variant, int sb_dtype, int act, const kqo_expert* e,
                    const float* x, float* out, int hidden, int inter, int gs,
                    float* scratch /* 3*inter */) {
    float* g = scratch;
    float* u = scratch + inter;
    float* a = scratch + 2 * inter;
    kqo_matvec_v(bits, variant, e->w[0], e->s[0], e->b[0], sb_dtype, x, g, inter, hidden, gs);
    kqo_matvec_v(bits, variant, e->w[1], e->s[1], e->b[1], sb_dtype, x, u, inter, hidden, gs);
    for (int i = 0; i < inter; i++) {
        float gv = g[i];
        if (act == 1) {
            float t = 0.7978845608f * (gv + 0.044715f * gv * gv * gv);
            a[i] = 0.5f * gv * (1.0f + tanhf(t)) * u[i];
        } else {
            a[i] = (gv / (1.0f + expf(-gv))) * u[i];
        }
    }
    kqo_matvec_v(bits, variant, e->w[2], e->s[2], e->b[2], sb_dtype, a, out, hidden, inter, gs);
}

/* Batched expert MLP over a stacked layer table:
 *   weights of expert e at  w[m] + e * wstride[m]  (bytes), same for s/b (elements)
 * x [T][hidden] fp32, idx [T][K] int32, out [T][K][hidden] fp32.
 * (t, k) pairs run in parallel with OpenMP when threads > 1. */
void kqo_moe_layer(int bits, int variant, int sb_dtype, int act, const void* const* w,
                   const int64_t* wstride,
                   const uint16_t* const* s, const uint16_t* const* b, const int64_t* sbstride,
                   const float* x, const int32_t* idx, int T, int K, float* out, int hidden,
                   int inter, int gs, int threads) {
    long total = (long)T * K;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
    for (long tk = 0; tk < total; tk++) {
        int t = (int)(tk / K);
        int e = idx[tk];
        kqo_expert ex;
        for (int m = 0; m < 3; m++) {
            ex.w[m] = (const uint8_t*)w[m] + (int64_t)e * wstride[m];
            ex.s[m] = s[m] + (int64_t)e * sbstride[m];
            ex.b[m] = b[m] + (int64_t)e * sbstride[m];
        }
        float* scratch = (float*)malloc(sizeof(float) * 3 * (size_t)inter);
        kqo_expert_mlp(bits, variant, sb_dtype, act, &ex, x + (size_t)t * hidden,
                       out + (size_t)tk * hidden, hidden, inter, gs, scratch);
        free(scratch);
    }
}

/* ---- router ----------------------------------------------------------------- */
/* softmax over E logits, then K rounds of argmax with strict '>' so the lowest
 * index wins a tie, then the K probabilities renormalised to sum to one.
 * Selection is done on the logits (softmax is monotone, so the order is the
 * same) so that ties are decided exactly rather than after exp() rounding. */
void kqo_router_topk(const float* logits, int T, int E, int K, int32_t* idx, float* w) {
    for (int t = 0; t < T; t++) {
        const float* l = logits + (size_t)t * E;
        float mx = -INFINITY;
        for (int i = 0; i < E; i++) mx = l[i] > mx ? l[i] : mx;
        unsigned char* taken = (unsigned char*)calloc((size_t)E, 1);
        float sel_e[64];
        float ssum = 0.0f;
        for (int k = 0; k < K; k++) {
            int best = -1;
            float bv = -INFINITY;
            for (int i = 0; i < E; i++) {
                if (!taken[i] && (best < 0 || l[i] > bv)) { best = i; bv = l[i]; }
            }
            taken[best] = 1;
            idx[(size_t)t * K + k] = best;
            sel_e[k] = expf(bv - mx);
            ssum += sel_e[k];
        }
        for (int k = 0; k < K; k++) w[(size_t)t * K + k] = sel_e[k] / ssum;
        free(taken);
    }
}

/* ---- combine ---------------------------------------------------------------- */
/* out[t][h] = [res[t][h]] + sum_k w[t][k] * y[t][k][h] [+ gate[t] * shared[t][h]] */
void kqo_combine(const float* y, const float* w, const float* res, const float* shared,
                 const float* gate, int T, int K, int H, float* out) {
    for (int t = 0; t < T; t++)
        for (int h = 0; h < H; h++) {
            float acc = 0.0f;
            for (int k = 0; k < K; k++) acc += y[((size_t)t * K + k) * H + h] * w[(size_t)t * K + k];
            /* blend_residual order: (res + expert_sum) + gate * shared */
            if (res) acc = res[(size_t)t * H + h] + acc;
            if (shared) acc = acc + shared[(size_t)t * H + h] * gate[t];
            out[(size_t)t * H + h] = acc;
        }
}

/* fp32 -> fp16 bits, round-to-nearest-even (the reference's float_to_half). */
void kqo_f32_to_f16(const float* in, uint16_t* out, long n) {
    for (long i = 0; i < n; i++) out[i] = kqo_to_f16(in[i]);
}
