// The chunked matrix products of the m-token path (prefill chunks, and one
// decode step of up to 64 sequences): Y[m x R] = X[m x K] . W[R x K]^T with
// W in the tile layout (Q4_0 / Q4_1 / Q8_0), m <= 64.
//
// The reference runs a prefill chunk as its fused q4 kernels over a z axis of
// tokens (fused.go:294-320, kernels_fused.go:28-73): every token re-reads the
// weights.  Here a CTA owns a tile of 64 tokens x 64 weight rows, stages one
// 32-column block of the activations and of the dequantised weights in
// shared memory per step, and each thread accumulates a 4 x 4 register tile,
// so a weight block is read once for all tokens of the chunk.  Weights are
// dequantised exactly (f16 scale times a small integer is exact in f32); the
// products are f32 FMAs, summed per block and then over blocks (cpu.go:143-222
// sums a block, then d * block over blocks).
//
// Few row tiles (e.g. 9 for a 576-row output) would leave most SMs idle, so
// the K range is split over the CTAs of a thread-block cluster (up to 8);
// each keeps its partial tile in shared memory, and after a cluster barrier
// each CTA adds the cluster's partials for its share of the tokens through
// distributed shared memory, in rank order (deterministic), and runs the
// epilogue: QKV bias + RoPE + q store + KV append, the residual add,
// SwiGLU, or per-token argmax partials for the vocabulary head.  The next
// K block's loads are issued before the current block's products.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>
#include <initializer_list>

#include "kernels.hpp"

namespace llmb {

namespace {

namespace cg = cooperative_groups;

constexpr int kTM = 64;    // tokens per CTA tile
constexpr int kTR = 64;    // weight rows per CTA tile (8 tiles of 8 rows)
constexpr int kXS = kTM + 4;  // shared row stride (floats) of the k-major staging arrays
constexpr int kGT = 256;   // threads

__device__ __forceinline__ float b2f(uint32_t v, int k) {
    return __int_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | k));
}

// Rows [0, rows) of the concatenated matrices mats[0..nm): the one holding
// global row g, and g's row within it.
struct MatSet {
    QMat m[3];
    int nm;
};

__device__ __forceinline__ int mat_of(const MatSet &ms, int g, int &local) {
    int base = 0;
    for (int j = 0; j < ms.nm; ++j) {
        if (g < base + ms.m[j].rows) {
            local = g - base;
            return j;
        }
        base += ms.m[j].rows;
    }
    local = 0;
    return ms.nm - 1;
}

// One thread's share of a weight block: row t / 4 of the tile, quarter t % 4
// of the block's quants (4 bytes of Q4, 8 of Q8), with its scale (and min).
struct WRegs {
    uint32_t w0, w1;
    float d, mn;
    bool valid;
};

__device__ __forceinline__ void load_w(const QMat &m, int r0, int kb, WRegs &R) {
    const int t = threadIdx.x, row = t >> 2, q = t & 3;
    const int g = r0 + row;
    R.valid = g < m.rows;
    if (!R.valid) return;
    const uint8_t *tile = m.tiles + (size_t)(g >> 3) * m.tile_bytes;
    const int r = g & 7;
    if (m.type == 8) {
        const uint2 w = __ldg(reinterpret_cast<const uint2 *>(tile + ((size_t)kb * 8 + r) * 32 + 8 * q));
        R.w0 = w.x, R.w1 = w.y;
        R.d = __half2float(__ldg(reinterpret_cast<const __half *>(tile + (size_t)m.nb * 256) + kb * 8 + r));
        return;
    }
    R.w0 = __ldg(reinterpret_cast<const uint32_t *>(tile + ((size_t)kb * 8 + r) * 16 + 4 * q));
    const __half *dp = reinterpret_cast<const __half *>(tile + (size_t)m.nb * 128);
    R.d = __half2float(__ldg(dp + kb * 8 + r));
    if (m.type == 3) R.mn = __half2float(__ldg(dp + (size_t)m.nb * 8 + kb * 8 + r));
}

// The block dequantised into ws[k][row] (k-major), exactly: Q4_0 d * (q - 8)
// (cpu.go:164-179), Q4_1 d * q + m (cpu.go:181-200), Q8_0 d * q
// (cpu.go:201-215); zero past the matrix's rows.
__device__ __forceinline__ void store_w(int type, const WRegs &R, float *ws) {
    const int t = threadIdx.x, row = t >> 2, q = t & 3;
    if (type == 8) {
        const uint32_t u0 = R.w0 ^ 0x80808080u, u1 = R.w1 ^ 0x80808080u;
        constexpr float off = 8388736.f;  // 2^23 + 128
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ws[(8 * q + i) * kXS + row] = R.valid ? R.d * (b2f(u0, i) - off) : 0.f;
            ws[(8 * q + 4 + i) * kXS + row] = R.valid ? R.d * (b2f(u1, i) - off) : 0.f;
        }
        return;
    }
    const uint32_t lo = R.w0 & 0x0F0F0F0Fu, hi = (R.w0 >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float a, b;
        if (type == 3) a = fmaf(R.d, b2f(lo, i) - 8388608.f, R.mn), b = fmaf(R.d, b2f(hi, i) - 8388608.f, R.mn);
        else a = R.d * (b2f(lo, i) - 8388616.f), b = R.d * (b2f(hi, i) - 8388616.f);
        ws[(4 * q + i) * kXS + row] = R.valid ? a : 0.f;
        ws[(4 * q + i + 16) * kXS + row] = R.valid ? b : 0.f;
    }
}

// X columns [32 kb, 32 kb + 32) of m tokens (row stride K): thread t holds
// token t / 4, 8 columns; tokens >= m are zero.
__device__ __forceinline__ void load_x(const float *x, int K, int m, int kb, float4 &a, float4 &b) {
    const int t = threadIdx.x, tok = t >> 2, c0 = (t & 3) * 8;
    a = b = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tok < m) {
        const float4 *p = reinterpret_cast<const float4 *>(x + (size_t)tok * K + kb * 32 + c0);
        a = __ldcg(p), b = __ldcg(p + 1);
    }
}

__device__ __forceinline__ void store_x(const float4 &a, const float4 &b, float *xs) {
    const int t = threadIdx.x, tok = t >> 2, c0 = (t & 3) * 8;
    xs[(c0 + 0) * kXS + tok] = a.x, xs[(c0 + 1) * kXS + tok] = a.y;
    xs[(c0 + 2) * kXS + tok] = a.z, xs[(c0 + 3) * kXS + tok] = a.w;
    xs[(c0 + 4) * kXS + tok] = b.x, xs[(c0 + 5) * kXS + tok] = b.y;
    xs[(c0 + 6) * kXS + tok] = b.z, xs[(c0 + 7) * kXS + tok] = b.w;
}

enum Epi { EPI_QKV = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

struct GemmArgs {
    const DevModel *dm;
    const TokBatch *tb;
    const float *x;      // [m][K]
    int m, nb;           // tokens, 32-column blocks of K
    MatSet a, b;         // b: the up matrix of SwiGLU (a: gate)
    int splits;          // the cluster's CTAs along K (1, 2, 4 or 8)
    int l;               // layer (QKV: which KV cache)
    float *out;          // RESID: x [m][E]; SWIGLU: act [m][F]
    int out_ld;
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// The epilogue of token t, rows r0 + 4 tx + c (c < 4) of the tile, whose
// local rows in matrix `seg` of ga.a start at la.
template <int EPI, int NM>
__device__ __forceinline__ void epilogue(const GemmArgs &ga, const DevModel &dm, const QMat &ma, int seg, int la,
                                         int r0, int t, int tx, const float (&v)[NM][4]) {
    if (t >= ga.m) return;
    if constexpr (EPI == EPI_RESID) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if (la + tx * 4 + c >= ma.rows) continue;
            float *p = ga.out + (size_t)t * ga.out_ld + r0 + tx * 4 + c;
            *p = __fadd_rn(__ldcg(p), v[0][c]);
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int row = r0 + tx * 4 + c;
            if (row >= dm.ff || row >= ma.rows) continue;
            const float g = v[0][c], u = v[NM - 1][c];
            const float den = __fadd_rn(1.f, (float)exp(-(double)g));  // cpu.go:345
            ga.out[(size_t)t * ga.out_ld + row] = __fmul_rn(__fdiv_rn(g, den), u);
        }
    } else if constexpr (EPI == EPI_QKV) {  // kernels_fused.go:212-224; cpu.go:279-303
        const int pos = ga.tb ? ga.tb->pos[t] : (int)dm.state[0] + t;
        const Layer &L = dm.layer[ga.l];
        const float *bias = seg == 0 ? L.bq : seg == 1 ? L.bk : L.bv;
        float o[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) o[c] = bias ? __fadd_rn(v[0][c], __ldg(bias + la + tx * 4 + c)) : v[0][c];
        if (seg < 2) {  // rotate adjacent pairs (cpu.go:371-385)
            const int hp = dm.head_dim >> 1;
#pragma unroll
            for (int c = 0; c < 4; c += 2) {
                const int p = ((la + tx * 4 + c) % dm.head_dim) >> 1;
                const float2 cs = __ldg(reinterpret_cast<const float2 *>(dm.rope_cs) + (size_t)pos * hp + p);
                const float e = o[c], f = o[c + 1];
                o[c] = __fsub_rn(__fmul_rn(e, cs.x), __fmul_rn(f, cs.y));
                o[c + 1] = __fadd_rn(__fmul_rn(e, cs.y), __fmul_rn(f, cs.x));
            }
        }
        float *kv = ga.tb ? ga.tb->kv + ((size_t)ga.tb->slot[t] * ga.tb->layers + ga.l) * 2 * (size_t)dm.ctx * dm.kvd
                          : L.kv;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int row = la + tx * 4 + c;
            if (seg == 0) dm.q[(size_t)t * dm.embd + row] = o[c];
            else if (seg == 1) kv[(size_t)pos * dm.kvd + row] = o[c];
            else kv[((size_t)dm.ctx + pos) * dm.kvd + row] = o[c];
        }
    }
}

__host__ __device__ constexpr size_t gemm_smem_floats(int nm) {
    const size_t stage = (size_t)(1 + nm) * 32 * kXS, part = (size_t)nm * kGT * 16;
    return stage > part ? stage : part;
}

// grid (row tiles, splits), cluster (1, splits, 1): CTA (rt, s) multiplies
// row tile rt over its share s of the K blocks; the cluster's CTAs
// then add their partial tiles through distributed shared memory, in rank
// order, each for its own share of the tokens, and run the epilogue.
template <int EPI>
__global__ void __launch_bounds__(kGT) k_gemm(const __grid_constant__ GemmArgs ga) {
    constexpr int NM = EPI == EPI_SWIGLU ? 2 : 1;
    __shared__ __align__(16) float sm[gemm_smem_floats(NM)];
    float *xs = sm, *wsm = sm + 32 * kXS;
    const DevModel &dm = *ga.dm;
    const int rt = blockIdx.x, sp = blockIdx.y, r0 = rt * kTR;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    int la = 0, lb = 0;
    const int seg = mat_of(ga.a, r0, la);
    const QMat &ma = ga.a.m[seg];
    const QMat &mb = ga.b.m[NM == 2 ? mat_of(ga.b, r0, lb) : 0];
    const int kb0 = ga.nb * sp / ga.splits, kb1 = ga.nb * (sp + 1) / ga.splits;  // balanced K share
    const int K = ga.nb * 32;
    float acc[NM][4][4];
#pragma unroll
    for (int j = 0; j < NM; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[j][i][c] = 0.f;
    WRegs wa{}, wb{};
    float4 xa, xb;
    if (kb0 < kb1) {
        load_w(ma, la, kb0, wa);
        if (NM == 2) load_w(mb, lb, kb0, wb);
        load_x(ga.x, K, ga.m, kb0, xa, xb);
    }
    for (int kb = kb0; kb < kb1; ++kb) {
        store_x(xa, xb, xs);
        store_w(ma.type, wa, wsm);
        if (NM == 2) store_w(mb.type, wb, wsm + 32 * kXS);
        __syncthreads();
        if (kb + 1 < kb1) {  // the next block's loads fly during this block's products
            load_w(ma, la, kb + 1, wa);
            if (NM == 2) load_w(mb, lb, kb + 1, wb);
            load_x(ga.x, K, ga.m, kb + 1, xa, xb);
        }
        // paired FMAs (two independent fused FMAs per instruction) over row pairs (c, c + 1)
        float2 blk[NM][4][2];
#pragma unroll
        for (int j = 0; j < NM; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) blk[j][i][0] = blk[j][i][1] = make_float2(0.f, 0.f);
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            const float4 a4 = *reinterpret_cast<const float4 *>(xs + k * kXS + ty * 4);
            const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
            for (int j = 0; j < NM; ++j) {
                const float4 b4 = *reinterpret_cast<const float4 *>(wsm + j * 32 * kXS + k * kXS + tx * 4);
                const float2 b01 = make_float2(b4.x, b4.y), b23 = make_float2(b4.z, b4.w);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 a2 = make_float2(av[i], av[i]);
                    blk[j][i][0] = __ffma2_rn(a2, b01, blk[j][i][0]);
                    blk[j][i][1] = __ffma2_rn(a2, b23, blk[j][i][1]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < NM; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[j][i][0] += blk[j][i][0].x, acc[j][i][1] += blk[j][i][0].y;
                acc[j][i][2] += blk[j][i][1].x, acc[j][i][3] += blk[j][i][1].y;
            }
        __syncthreads();
    }
    if constexpr (EPI == EPI_ARGMAX) {  // no split: the tile's best row per token
        __shared__ float bvs[kTM][16];
        __shared__ int bis[kTM][16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float bv = -FLT_MAX;
            int bi = 0x7fffffff;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int row = r0 + tx * 4 + c;
                if (row < dm.vocab && better(acc[0][i][c], row, bv, bi)) bv = acc[0][i][c], bi = row;
            }
            bvs[ty * 4 + i][tx] = bv, bis[ty * 4 + i][tx] = bi;
        }
        __syncthreads();
        if (threadIdx.x < ga.m) {
            float bv = -FLT_MAX;
            int bi = 0x7fffffff;
            for (int c = 0; c < 16; ++c)
                if (better(bvs[threadIdx.x][c], bis[threadIdx.x][c], bv, bi)) bv = bvs[threadIdx.x][c], bi = bis[threadIdx.x][c];
            dm.gam[(size_t)threadIdx.x * gridDim.x + rt] = make_float2(bv, __int_as_float(bi));
        }
    } else {
        if (ga.splits == 1) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float v[NM][4];
#pragma unroll
                for (int j = 0; j < NM; ++j)
#pragma unroll
                    for (int c = 0; c < 4; ++c) v[j][c] = acc[j][i][c];
                epilogue<EPI, NM>(ga, dm, ma, seg, la, r0, ty * 4 + i, tx, v);
            }
            return;
        }
        // partial tile into this CTA's shared memory: unit (j, i, thread) is a float4 of 4 rows
#pragma unroll
        for (int j = 0; j < NM; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                *reinterpret_cast<float4 *>(sm + ((size_t)(j * 4 + i) * kGT + threadIdx.x) * 4) =
                    make_float4(acc[j][i][0], acc[j][i][1], acc[j][i][2], acc[j][i][3]);
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
        // CTA s finishes the source threads [s * 256 / S, (s + 1) * 256 / S) (a range of token groups ty)
        const int S = ga.splits, per = kGT / S;
        for (int u = threadIdx.x; u < per * 4; u += kGT) {
            const int src = sp * per + (u >> 2), i = u & 3;
            float v[NM][4];
#pragma unroll
            for (int j = 0; j < NM; ++j) v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.f;
            for (int r = 0; r < S; ++r) {
                const float *rs = cl.map_shared_rank(sm, r);
#pragma unroll
                for (int j = 0; j < NM; ++j) {
                    const float4 p = *reinterpret_cast<const float4 *>(rs + ((size_t)(j * 4 + i) * kGT + src) * 4);
                    v[j][0] += p.x, v[j][1] += p.y, v[j][2] += p.z, v[j][3] += p.w;
                }
            }
            epilogue<EPI, NM>(ga, dm, ma, seg, la, r0, (src >> 4) * 4 + i, src & 15, v);
        }
        cl.sync();  // the partials stay readable until every CTA of the cluster is done with them
    }
}

// RMSNorm rows for the products (cpu.go:81-98): h[t] = (x[row t] * s) * w,
// s = 1 / sqrt(mean of squares + eps) in double; one CTA per token.
__global__ void __launch_bounds__(kGT) k_norm_rows(const DevModel *__restrict__ dmp, const float *w, const int *rows,
                                                   int row0) {
    const DevModel &dm = *dmp;
    const int t = blockIdx.x, E = dm.embd;
    const int src = rows ? rows[t] : row0 + t;
    const float *x = dm.x + (size_t)src * E;
    __shared__ float red[kGT / 32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < E; i += kGT) {
        const float v = __ldcg(x + i);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int k = 0; k < kGT / 32; ++k) ss += red[k];
    const float s = (float)(1.0 / sqrt((double)__fadd_rn(__fdiv_rn(ss, (float)E), dm.eps)));
    for (int i = threadIdx.x; i < E; i += kGT) dm.h[(size_t)t * E + i] = __fmul_rn(__fmul_rn(__ldcg(x + i), s), __ldg(w + i));
}

// The argmax of each token over the head's row-tile partials (first index of
// the largest value), into tb->out[t].
__global__ void __launch_bounds__(kGT) k_argmax_rows(const DevModel *__restrict__ dmp, TokBatch *tb, int parts) {
    const DevModel &dm = *dmp;
    const int t = blockIdx.x;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < parts; i += kGT) {
        const float2 p = __ldcg(dm.gam + (size_t)t * parts + i);
        const int pi = __float_as_int(p.y);
        if (better(p.x, pi, bv, bi)) bv = p.x, bi = pi;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    __shared__ float wv[kGT / 32];
    __shared__ int wi[kGT / 32];
    if ((threadIdx.x & 31) == 0) wv[threadIdx.x >> 5] = bv, wi[threadIdx.x >> 5] = bi;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kGT / 32; ++w)
            if (better(wv[w], wi[w], bv, bi)) bv = wv[w], bi = wi[w];
        tb->out[t] = bi == 0x7fffffff ? 0 : bi;
    }
}

MatSet mats(std::initializer_list<const QMat *> ms) {
    MatSet s{};
    for (const QMat *m : ms) s.m[s.nm++] = *m;
    return s;
}

// CTAs along K per row tile: the largest of 8, 4, 2 that keeps the grid
// within two CTAs per SM and gives each at least 2 K blocks.
int splits_for(int row_tiles, int nb, int nsm) {
    for (int s = 8; s > 1; s /= 2)
        if (row_tiles * s <= 2 * nsm && nb >= 2 * s) return s;
    return 1;
}

template <int EPI>
cudaError_t gemm(const GemmArgs &base, int rows, int nsm, cudaStream_t st) {
    GemmArgs ga = base;
    const int row_tiles = (rows + kTR - 1) / kTR;
    ga.splits = EPI == EPI_ARGMAX ? 1 : splits_for(row_tiles, ga.nb, nsm);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(row_tiles, ga.splits);
    cfg.blockDim = dim3(kGT);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = ga.splits, attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_gemm<EPI>, ga);
}

}  // namespace

cudaError_t launch_layer_mm(const DevModel *dm, const DevModel &hd, const Shapes &s, int l, int m, int nsm,
                            cudaStream_t st, const TokBatch *tb) {
    const Layer &L = hd.layer[l];
    const int E = s.embd, F = s.ff;
    GemmArgs ga{};
    ga.dm = dm, ga.tb = tb, ga.m = m, ga.l = l;
    // QKV
    k_norm_rows<<<m, kGT, 0, st>>>(dm, L.attn_norm, nullptr, 0);
    ga.x = hd.h, ga.nb = E / 32, ga.a = mats({&L.q, &L.k, &L.v});
    cudaError_t e = gemm<EPI_QKV>(ga, L.q.rows + L.k.rows + L.v.rows, nsm, st);
    // attention (per token, per head and chunk of 64 positions)
    launch_attention(dm, s, l, m, st, tb);
    // x += Wo att
    ga.x = hd.att, ga.nb = E / 32, ga.a = mats({&L.o}), ga.out = hd.x, ga.out_ld = E;
    if (e == cudaSuccess) e = gemm<EPI_RESID>(ga, L.o.rows, nsm, st);
    // act = SwiGLU(Wgate h, Wup h)
    k_norm_rows<<<m, kGT, 0, st>>>(dm, L.ffn_norm, nullptr, 0);
    ga.x = hd.h, ga.nb = E / 32, ga.a = mats({&L.gate}), ga.b = mats({&L.up}), ga.out = hd.act, ga.out_ld = F;
    if (e == cudaSuccess) e = gemm<EPI_SWIGLU>(ga, L.gate.rows, nsm, st);
    // x += Wdown act
    ga.x = hd.act, ga.nb = F / 32, ga.a = mats({&L.down}), ga.b = MatSet{}, ga.out = hd.x, ga.out_ld = E;
    if (e == cudaSuccess) e = gemm<EPI_RESID>(ga, L.down.rows, nsm, st);
    return e;
}

cudaError_t launch_head_mm(const DevModel *dm, const DevModel &hd, const Shapes &s, TokBatch *tb, const int *rows_dev,
                           int rows, int nsm, cudaStream_t st) {
    k_norm_rows<<<rows, kGT, 0, st>>>(dm, hd.out_norm, rows_dev, 0);
    GemmArgs ga{};
    ga.dm = dm, ga.tb = tb, ga.m = rows, ga.x = hd.h, ga.nb = s.embd / 32, ga.a = mats({&hd.head});
    const cudaError_t e = gemm<EPI_ARGMAX>(ga, hd.head.rows, nsm, st);
    k_argmax_rows<<<rows, kGT, 0, st>>>(dm, tb, (hd.head.rows + kTR - 1) / kTR);
    return e;
}


}  // namespace llmb
