// kq_table.cu -- HBM-resident quantized tables: layout, repack from the MLX
// layout (device), exact unpack back to it, and BKEX layer-file loading.
//
// An expert occupies, in this order:
//   gate/up pair matrix : (I/8) row-tiles x ceil(H/512) column tiles; each tile
//                         holds gate rows 8rt..8rt+7 (MMA rows 0-7) and up rows
//                         8rt..8rt+7 (MMA rows 8-15), so one pass yields both
//                         projections of the same intermediate rows
//   down matrix         : (H/16) row-tiles x ceil(I/512) column tiles
// Experts of a layer are contiguous; layers are contiguous.  With H and I
// multiples of 512 the expert is exactly as large as its MLX/BKEX form
// (e.g. 1,376,256 B for H2048/I512 3-bit).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "kq_internal.h"

namespace kq {

// ---- repack: MLX layout -> KQ tiles ---------------------------------------------
struct MlxSrc {
    const uint8_t* w;
    const uint16_t* s;
    const uint16_t* b;
    int64_t wstride, sbstride;  // bytes per expert
};

struct RepackArgs {
    MlxSrc a, b;      // b used only in pair mode
    uint8_t* dst;     // expert 0 of the destination matrix
    int64_t dst_stride;
    int bits, rows, cols, nrt, nst, pair, nexp;
};

__device__ __forceinline__ int mlx_code(const uint8_t* row, int bits, int i) {
    if (bits == 4) {
        uint32_t wv = reinterpret_cast<const uint32_t*>(row)[i >> 3];
        return (int)((wv >> (4 * (i & 7))) & 15u);
    }
    const int bit = 3 * i;
    uint32_t v = row[bit >> 3];
    if ((bit & 7) > 5) v |= (uint32_t)row[(bit >> 3) + 1] << 8;
    return (int)((v >> (bit & 7)) & 7u);
}

// MMA row m (0..15) of row-tile rt -> (source, row); pair mode interleaves a/b.
__device__ __forceinline__ void src_row(const RepackArgs& A, int rt, int m, int& which, int& row) {
    if (A.pair) {
        which = m >> 3;
        row = rt * 8 + (m & 7);
    } else {
        which = 0;
        row = rt * 16 + m;
    }
}

__global__ void repack_kernel(RepackArgs A) {
    const int W = A.bits == 3 ? 6 : 8;
    const int words_per_lane = 4 * W + 4;
    const int words_per_tile = 32 * words_per_lane;
    const long total = (long)A.nexp * A.nrt * A.nst * words_per_tile;
    const int ncols_row = A.cols;
    const int ngroups = A.cols / GS;
    const int64_t row_bytes = A.bits == 3 ? (int64_t)A.cols * 3 / 8 : (int64_t)A.cols / 2;
    for (long gid = blockIdx.x * (long)blockDim.x + threadIdx.x; gid < total;
         gid += (long)gridDim.x * blockDim.x) {
        const int wi = (int)(gid % words_per_tile);
        const long tile = gid / words_per_tile;
        const int st = (int)(tile % A.nst);
        const int rt = (int)((tile / A.nst) % A.nrt);
        const int e = (int)(tile / ((long)A.nst * A.nrt));
        const int lane = wi / words_per_lane, q = wi % words_per_lane;
        uint32_t word = 0;
        if (q < 4 * W) {
            const int set = q / W, w = q % W;
            const int m = (lane >> 2) + (set >= 2 ? 8 : 0);
            const int g8 = (lane & 3) + ((set & 1) ? 4 : 0);
            const int grp = st * TILE_GROUPS + g8;
            int which, row;
            src_row(A, rt, m, which, row);
            const MlxSrc& S = which ? A.b : A.a;
            const uint8_t* rowp = S.w + (int64_t)e * S.wstride + (int64_t)row * row_bytes;
            auto code = [&](int ci) -> uint32_t {
                const int col = grp * GS + ci;
                return (grp < ngroups && col < ncols_row) ? (uint32_t)mlx_code(rowp, A.bits, col) : 0u;
            };
            if (A.bits == 3) {
                for (int s = 0; s < 5; ++s) {
                    const int j = 5 * w + s;
                    word |= code(2 * j) << (3 * s);
                    word |= code(2 * j + 1) << (16 + 3 * s);
                }
                const int pj = 30 + w / 3, bitn = w % 3;
                word |= ((code(2 * pj) >> bitn) & 1u) << 15;
                word |= ((code(2 * pj + 1) >> bitn) & 1u) << 31;
            } else {
                for (int s = 0; s < 4; ++s) {
                    const int j = 4 * w + s;
                    word |= code(2 * j) << (4 * s);
                    word |= code(2 * j + 1) << (16 + 4 * s);
                }
            }
        } else {
            const int k = q - 4 * W;
            const int m = (lane >> 2) + (k >= 2 ? 8 : 0);
            const int grp = st * TILE_GROUPS + 2 * (lane & 3) + (k & 1);
            int which, row;
            src_row(A, rt, m, which, row);
            const MlxSrc& S = which ? A.b : A.a;
            if (grp < ngroups) {
                const int64_t off = (int64_t)e * (S.sbstride / 2) + (int64_t)row * ngroups + grp;
                word = (uint32_t)S.s[off] | ((uint32_t)S.b[off] << 16);
            }
        }
        const int chunk_q = q;  // lane word index: chunk q/4, position q%4
        uint8_t* tp = A.dst + (int64_t)e * A.dst_stride +
                      ((int64_t)rt * A.nst + st) * tile_bytes(A.bits);
        *reinterpret_cast<uint32_t*>(tp + tile_word_offset(lane, chunk_q)) = word;
    }
}

// ---- unpack: KQ tiles -> MLX layout ---------------------------------------------
struct UnpackArgs {
    const uint8_t* src;  // tiles of the matrix (one expert)
    uint8_t* w;
    uint16_t* s;
    uint16_t* b;
    int bits, rows, cols, nst, pair, which;  // which: 0 = a (gate/plain), 1 = b (up)
};

__device__ __forceinline__ uint32_t kq_word(const UnpackArgs& U, int rt, int st, int lane, int q) {
    const uint8_t* tp = U.src + ((int64_t)rt * U.nst + st) * tile_bytes(U.bits);
    return *reinterpret_cast<const uint32_t*>(tp + tile_word_offset(lane, q));
}

__device__ __forceinline__ void dst_tile(const UnpackArgs& U, int row, int& rt, int& m) {
    if (U.pair) {
        rt = row / 8;
        m = (row % 8) + (U.which ? 8 : 0);
    } else {
        rt = row / 16;
        m = row % 16;
    }
}

__device__ int kq_code(const UnpackArgs& U, int row, int col) {
    int rt, m;
    dst_tile(U, row, rt, m);
    const int st = col / TILE_COLS;
    const CodeLoc L = code_loc(m, col % TILE_COLS);
    const int W = U.bits == 3 ? 6 : 8;
    if (U.bits == 3) {
        if (L.pair < 30) {
            const int w = L.pair / 5, s = L.pair % 5;
            return (int)((kq_word(U, rt, st, L.lane, L.set * W + w) >> (3 * s + 16 * L.hi)) & 7u);
        }
        const int base = (L.pair - 30) * 3;
        int v = 0;
        for (int bb = 0; bb < 3; ++bb)
            v |= (int)((kq_word(U, rt, st, L.lane, L.set * W + base + bb) >> (15 + 16 * L.hi)) & 1u) << bb;
        return v;
    }
    const int w = L.pair / 4, s = L.pair % 4;
    return (int)((kq_word(U, rt, st, L.lane, L.set * W + w) >> (4 * s + 16 * L.hi)) & 15u);
}

__global__ void unpack_kernel(UnpackArgs U) {
    const int packs = U.cols / 8;  // 8 codes per pack
    const long total = (long)U.rows * packs;
    for (long gid = blockIdx.x * (long)blockDim.x + threadIdx.x; gid < total;
         gid += (long)gridDim.x * blockDim.x) {
        const int row = (int)(gid / packs), p = (int)(gid % packs);
        uint32_t word = 0;
        for (int t = 0; t < 8; ++t)
            word |= (uint32_t)kq_code(U, row, p * 8 + t) << ((U.bits == 3 ? 3 : 4) * t);
        if (U.bits == 3) {
            uint8_t* o = U.w + (int64_t)row * (U.cols * 3 / 8) + p * 3;
            o[0] = word & 0xFF;
            o[1] = (word >> 8) & 0xFF;
            o[2] = (word >> 16) & 0xFF;
        } else {
            reinterpret_cast<uint32_t*>(U.w)[(int64_t)row * packs + p] = word;
        }
    }
    const int ng = U.cols / GS;
    const long tsb = (long)U.rows * ng;
    for (long gid = blockIdx.x * (long)blockDim.x + threadIdx.x; gid < tsb;
         gid += (long)gridDim.x * blockDim.x) {
        const int row = (int)(gid / ng), g = (int)(gid % ng);
        int rt, m;
        dst_tile(U, row, rt, m);
        const int st = g / TILE_GROUPS, g8 = g % TILE_GROUPS;
        const int lane = (m & 7) * 4 + (g8 >> 1);
        const int k = ((m >> 3) << 1) | (g8 & 1);
        const int W = U.bits == 3 ? 6 : 8;
        const uint32_t v = kq_word(U, rt, st, lane, 4 * W + k);
        U.s[gid] = (uint16_t)(v & 0xFFFFu);
        U.b[gid] = (uint16_t)(v >> 16);
    }
}

}  // namespace kq

using namespace kq;

// ---- table -------------------------------------------------------------------------

static int check_desc(const kq_table_desc* d) {
    if (!d) return KQ_ERR_ARG;
    if (d->bits != 3 && d->bits != 4) return KQ_ERR_UNSUPPORTED;
    if (d->group_size != 64) return KQ_ERR_UNSUPPORTED;
    if (d->sb_dtype != KQ_DT_F16 && d->sb_dtype != KQ_DT_BF16) return KQ_ERR_ARG;
    if (d->activation != KQ_ACT_SILU && d->activation != KQ_ACT_GELU_TANH) return KQ_ERR_ARG;
    if (d->num_layers <= 0 || d->num_experts <= 0) return KQ_ERR_ARG;
    if (d->hidden <= 0 || d->inter <= 0 || d->hidden % 64 || d->inter % 64) return KQ_ERR_ARG;
    if (d->hidden % 16 || d->inter % 8) return KQ_ERR_ARG;
    return KQ_OK;
}

extern "C" int kq_table_create(const kq_table_desc* desc, kq_table** out) {
    if (!out) return KQ_ERR_ARG;
    *out = nullptr;
    int rc = check_desc(desc);
    if (rc) return rc;
    kq_table* t = new (std::nothrow) kq_table();
    if (!t) return KQ_ERR_ALLOC;
    t->d = *desc;
    t->tb = tile_bytes(desc->bits);
    t->nst_h = (desc->hidden + TILE_COLS - 1) / TILE_COLS;
    t->nst_i = (desc->inter + TILE_COLS - 1) / TILE_COLS;
    t->i8 = desc->inter / 8;
    t->h16 = desc->hidden / 16;
    t->gateup_bytes = (size_t)t->i8 * t->nst_h * t->tb;
    t->down_bytes = (size_t)t->h16 * t->nst_i * t->tb;
    t->expert_bytes = t->gateup_bytes + t->down_bytes;
    t->layer_bytes = t->expert_bytes * desc->num_experts;
    t->bytes = t->layer_bytes * desc->num_layers;
    if (cudaMalloc(&t->base, t->bytes) != cudaSuccess) {
        cudaGetLastError();
        delete t;
        return KQ_ERR_ALLOC;
    }
    if (cudaMemset(t->base, 0, t->bytes) != cudaSuccess) {
        cudaFree(t->base);
        delete t;
        return KQ_ERR_CUDA;
    }
    *out = t;
    return KQ_OK;
}

extern "C" int kq_table_destroy(kq_table* t) {
    if (!t) return KQ_OK;
    if (t->base) cudaFree(t->base);
    delete t;
    return KQ_OK;
}

extern "C" int kq_table_desc_get(const kq_table* t, kq_table_desc* desc) {
    if (!t || !desc) return KQ_ERR_ARG;
    *desc = t->d;
    return KQ_OK;
}

extern "C" size_t kq_table_bytes(const kq_table* t) { return t ? t->bytes : 0; }
extern "C" size_t kq_table_expert_bytes(const kq_table* t) { return t ? t->expert_bytes : 0; }

static int launch_repack(const RepackArgs& A, cudaStream_t s) {
    const int W = A.bits == 3 ? 6 : 8;
    const long total = (long)A.nexp * A.nrt * A.nst * 32 * (4 * W + 4);
    const int threads = 256;
    const long blocks = std::min<long>((total + threads - 1) / threads, 148L * 64);
    repack_kernel<<<(unsigned)blocks, threads, 0, s>>>(A);
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

static MlxSrc to_src(const kq_mlx_matrix* m) {
    MlxSrc s;
    s.w = static_cast<const uint8_t*>(m->weight);
    s.s = static_cast<const uint16_t*>(m->scales);
    s.b = static_cast<const uint16_t*>(m->biases);
    s.wstride = m->weight_stride;
    s.sbstride = m->sb_stride;
    return s;
}

extern "C" int kq_table_load_mlx(kq_table* t, int layer, int expert_begin, int num_experts,
                                 const kq_mlx_matrix* gate, const kq_mlx_matrix* up,
                                 const kq_mlx_matrix* down, void* stream) {
    if (!t || !gate || !up || !down) return KQ_ERR_ARG;
    if (layer < 0 || layer >= t->d.num_layers) return KQ_ERR_ARG;
    if (expert_begin < 0 || num_experts <= 0 || expert_begin + num_experts > t->d.num_experts)
        return KQ_ERR_ARG;
    if (!gate->weight || !gate->scales || !gate->biases || !up->weight || !up->scales ||
        !up->biases || !down->weight || !down->scales || !down->biases)
        return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t* ebase = t->base + (size_t)layer * t->layer_bytes + (size_t)expert_begin * t->expert_bytes;
    RepackArgs A{};
    A.a = to_src(gate);
    A.b = to_src(up);
    A.dst = ebase;
    A.dst_stride = (int64_t)t->expert_bytes;
    A.bits = t->d.bits;
    A.rows = 2 * t->d.inter;
    A.cols = t->d.hidden;
    A.nrt = t->i8;
    A.nst = t->nst_h;
    A.pair = 1;
    A.nexp = num_experts;
    int rc = launch_repack(A, s);
    if (rc) return rc;
    RepackArgs D{};
    D.a = to_src(down);
    D.b = D.a;
    D.dst = ebase + t->gateup_bytes;
    D.dst_stride = (int64_t)t->expert_bytes;
    D.bits = t->d.bits;
    D.rows = t->d.hidden;
    D.cols = t->d.inter;
    D.nrt = t->h16;
    D.nst = t->nst_i;
    D.pair = 0;
    D.nexp = num_experts;
    return launch_repack(D, s);
}

extern "C" int kq_table_unpack_mlx(const kq_table* t, int layer, int expert, int matrix,
                                   void* weight, void* scales, void* biases, void* stream) {
    if (!t || !weight || !scales || !biases) return KQ_ERR_ARG;
    if (layer < 0 || layer >= t->d.num_layers || expert < 0 || expert >= t->d.num_experts)
        return KQ_ERR_ARG;
    if (matrix < 0 || matrix > 2) return KQ_ERR_ARG;
    const uint8_t* ebase = t->base + (size_t)layer * t->layer_bytes + (size_t)expert * t->expert_bytes;
    UnpackArgs U{};
    U.bits = t->d.bits;
    U.w = static_cast<uint8_t*>(weight);
    U.s = static_cast<uint16_t*>(scales);
    U.b = static_cast<uint16_t*>(biases);
    if (matrix < 2) {
        U.src = ebase;
        U.rows = t->d.inter;
        U.cols = t->d.hidden;
        U.nst = t->nst_h;
        U.pair = 1;
        U.which = matrix;
    } else {
        U.src = ebase + t->gateup_bytes;
        U.rows = t->d.hidden;
        U.cols = t->d.inter;
        U.nst = t->nst_i;
        U.pair = 0;
        U.which = 0;
    }
    const long total = (long)U.rows * (U.cols / 8);
    const int threads = 256;
    const long blocks = std::min<long>((total + threads - 1) / threads, 148L * 32);
    unpack_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(U);
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

// ---- dense matrices ---------------------------------------------------------------------

extern "C" int kq_qmat_load_mlx(kq_qmat* m, const kq_mlx_matrix* a, const kq_mlx_matrix* b,
                                void* stream) {
    if (!m || !a || !a->weight || !a->scales || !a->biases) return KQ_ERR_ARG;
    if (m->pair && (!b || !b->weight || !b->scales || !b->biases)) return KQ_ERR_ARG;
    RepackArgs A{};
    A.a = to_src(a);
    A.b = m->pair ? to_src(b) : A.a;
    A.dst = m->base;
    A.dst_stride = 0;
    A.bits = m->bits;
    A.rows = m->pair ? 2 * m->rows : m->rows;
    A.cols = m->cols;
    A.nrt = m->nrt;
    A.nst = m->nst;
    A.pair = m->pair;
    A.nexp = 1;
    return launch_repack(A, static_cast<cudaStream_t>(stream));
}

extern "C" int kq_qmat_unpack_mlx(const kq_qmat* m, int which, void* weight, void* scales,
                                  void* biases, void* stream) {
    if (!m || !weight || !scales || !biases) return KQ_ERR_ARG;
    if (which < 0 || which > (m->pair ? 1 : 0)) return KQ_ERR_ARG;
    UnpackArgs U{};
    U.src = m->base;
    U.w = static_cast<uint8_t*>(weight);
    U.s = static_cast<uint16_t*>(scales);
    U.b = static_cast<uint16_t*>(biases);
    U.bits = m->bits;
    U.rows = m->rows;
    U.cols = m->cols;
    U.nst = m->nst;
    U.pair = m->pair;
    U.which = which;
    const long total = (long)U.rows * (U.cols / 8);
    const long blocks = std::min<long>((total + 255) / 256, 148L * 32);
    unpack_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(U);
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

// ---- BKEX -----------------------------------------------------------------------------

int kq::bkex_parse(const uint8_t* hdr, size_t n, BkexInfo* info) {
    if (n < 4096 || memcmp(hdr, "BKEX", 4) != 0) return KQ_ERR_FORMAT;
    uint32_t version, ne, nt;
    uint64_t esz;
    memcpy(&version, hdr + 4, 4);
    memcpy(&ne, hdr + 8, 4);
    memcpy(&esz, hdr + 12, 8);
    memcpy(&nt, hdr + 20, 4);
    if (nt != 9 || ne == 0 || esz == 0) return KQ_ERR_FORMAT;
    static const char* names[9] = {"gate_proj.weight", "gate_proj.scales", "gate_proj.biases",
                                   "up_proj.weight",   "up_proj.scales",   "up_proj.biases",
                                   "down_proj.weight", "down_proj.scales", "down_proj.biases"};
    memset(info, 0, sizeof(*info));
    info->num_experts = (int)ne;
    info->expert_size = esz;
    int pos = 24;
    int found = 0;
    for (uint32_t i = 0; i < nt; ++i) {
        uint8_t nl = hdr[pos];
        char nm[25] = {0};
        memcpy(nm, hdr + pos + 1, nl < 24 ? nl : 24);
        uint32_t off, nb, d0, d1;
        memcpy(&off, hdr + pos + 25, 4);
        memcpy(&nb, hdr + pos + 29, 4);
        memcpy(&d0, hdr + pos + 33, 4);
        memcpy(&d1, hdr + pos + 37, 4);
        uint8_t dt = hdr[pos + 41];
        pos += 42;
        for (int k = 0; k < 9; ++k)
            if (strcmp(nm, names[k]) == 0) {
                info->off[k] = off;
                info->nbytes[k] = nb;
                info->d0[k] = d0;
                info->d1[k] = d1;
                info->dtype[k] = dt;
                found |= 1 << k;
            }
    }
    if (found != 0x1FF) return KQ_ERR_FORMAT;
    info->inter = (int)info->d0[0];
    info->hidden = (int)info->d1[1] * 64;
    if (info->inter <= 0 || info->hidden <= 0) return KQ_ERR_FORMAT;
    // bits from the gate weight bytes (kandiga/metal/kandiga_cpu_expert_lg.m:98-107)
    const uint64_t expect4 = (uint64_t)info->inter * info->hidden / 2;
    info->bits = info->nbytes[0] < expect4 ? 3 : 4;
    info->sb_dtype = info->dtype[1] == 1 ? KQ_DT_BF16 : KQ_DT_F16;
    // GELU-tanh for expert_dim 704 (kandiga/metal/kandiga_cpu_expert_lg.m:109-111)
    info->activation = info->inter == 704 ? KQ_ACT_GELU_TANH : KQ_ACT_SILU;
    return KQ_OK;
}

extern "C" int kq_table_load_bkex(kq_table* t, int layer, const void* file_bytes, size_t nbytes,
                                  void* stream) {
    if (!t || !file_bytes) return KQ_ERR_ARG;
    BkexInfo info;
    int rc = bkex_parse(static_cast<const uint8_t*>(file_bytes), nbytes, &info);
    if (rc) return rc;
    if (info.hidden != t->d.hidden || info.inter != t->d.inter || info.bits != t->d.bits ||
        info.num_experts > t->d.num_experts || info.sb_dtype != t->d.sb_dtype)  // experts [0, file's) are filled
        return KQ_ERR_FORMAT;
    if (nbytes < 4096 + (size_t)info.num_experts * info.expert_size) return KQ_ERR_FORMAT;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int chunk = 32;
    uint8_t* staging = nullptr;
    const size_t stage_bytes = (size_t)chunk * info.expert_size;
    if (cudaMalloc(&staging, stage_bytes) != cudaSuccess) {
        cudaGetLastError();
        return KQ_ERR_ALLOC;
    }
    const uint8_t* payload = static_cast<const uint8_t*>(file_bytes) + 4096;
    for (int e0 = 0; e0 < info.num_experts && rc == KQ_OK; e0 += chunk) {
        const int n = std::min(chunk, info.num_experts - e0);
        if (cudaMemcpyAsync(staging, payload + (size_t)e0 * info.expert_size,
                            (size_t)n * info.expert_size, cudaMemcpyHostToDevice, s) != cudaSuccess) {
            rc = KQ_ERR_CUDA;
            break;
        }
        kq_mlx_matrix m[3];
        for (int k = 0; k < 3; ++k) {
            m[k].weight = staging + info.off[3 * k];
            m[k].scales = staging + info.off[3 * k + 1];
            m[k].biases = staging + info.off[3 * k + 2];
            m[k].weight_stride = (int64_t)info.expert_size;
            m[k].sb_stride = (int64_t)info.expert_size;
        }
        rc = kq_table_load_mlx(t, layer, e0, n, &m[0], &m[1], &m[2], stream);
        if (rc == KQ_OK && cudaStreamSynchronize(s) != cudaSuccess) rc = KQ_ERR_CUDA;
    }
    cudaFree(staging);
    return rc;
}

#include <map>
#include <mutex>
#include <utility>

cudaError_t kq::raise_smem_limit(const void* kernel, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> limits;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    size_t& cur = limits[{kernel, dev}];
    if (cur >= bytes) return cudaSuccess;
    const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err == cudaSuccess) cur = bytes;
    return err;
}
