// The chunked matrix products of the m-token path (prefill chunks, and one
// decode step of up to 64 sequences): Y[m x R] = X[m x K] . W[R x K]^T with
// W in the tile layout (Q4_0 / Q4_1 / Q8_0), m <= 64.
//
// The reference runs a prefill chunk as its fused q4 kernels over a z axis of
// tokens (fused.go:294-320, kernels_fused.go:28-73): every token re-reads the
// weights.  Here a weight block is read once for all tokens of the chunk, in
// one of two kernels:
//
//   k_mma (the default): the tensor cores.  A CTA owns 128 weight rows x 64
//   tokens; each 32-column block of the weights (dequantised exactly in f32)
//   and of the activations is split exactly into bf16 pieces, and the piece
//   products that reach 2^-18 of a x run as tcgen05.mma with f32
//   accumulators in tensor memory.
//
//   k_gemm (an A/B path): the FP32 CUDA cores.  A CTA owns 64 tokens x 64
//   weight rows and each thread accumulates a 4 x 4 register tile of f32
//   FMAs, summed per block and then over blocks (cpu.go:143-222 sums a block,
//   then d * block over blocks).
//
// Few row tiles (e.g. 5 for a 576-row output) would leave most SMs idle, so
// the K range is split over the CTAs of a thread-block cluster (up to 8 for
// k_gemm, 16 for k_mma); each keeps its partial tile in shared memory, and
// after a cluster barrier each CTA adds the cluster's partials for its share
// of the tokens through distributed shared memory, in rank order
// (deterministic), and runs the epilogue: QKV bias + RoPE + q store + KV
// append, the residual add, SwiGLU, or per-token argmax partials for the
// vocabulary head.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>
#include <initializer_list>
#include <mutex>
#include <utility>

#include "kernels.hpp"

namespace llmb {

namespace {

namespace cg = cooperative_groups;

constexpr int kTM = 64;    // tokens per CTA tile
constexpr int kTR = 64;    // weight rows per CTA tile (8 tiles of 8 rows)
constexpr int kXS = kTM + 4;  // shared row stride (floats) of the k-major staging arrays
constexpr int kGT = 256;   // threads
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float b2f(uint32_t v, int k) {
    return __int_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | k));
}

// Rows [0, rows) of the concatenated matrices mats[0..nm): the one holding
// global row g, and g's row within it.
struct MatSet {
    QMat m[3];
    int nm;
};

// (Unrolled over the 3 slots, so that the descriptors are read at fixed
// offsets of the kernel parameter, not through a computed address.)
__device__ __forceinline__ int mat_of(const MatSet &ms, int g, int &local) {
    int base = 0;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        if (j < ms.nm && g < base + ms.m[j].rows) {
            local = g - base;
            return j;
        }
        if (j < ms.nm) base += ms.m[j].rows;
    }
    local = 0;
    return ms.nm - 1;
}

// Descriptor j of a set, read at a fixed offset (see mat_of).
__device__ __forceinline__ const QMat &mat_at(const MatSet &ms, int j) {
    return j == 0 ? ms.m[0] : j == 1 ? ms.m[1] : ms.m[2];
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
    int splits;          // the cluster's CTAs along K (1, 2, 4 or 8; 1-16 for the tensor-core products)
    int l;               // layer (QKV: which KV cache)
    float *out;          // RESID: x [m][E]; SWIGLU: act [m][F]
    int out_ld;
    // k_mma only: with norm_w, x is the raw residual and the product reads RMSNorm(x) * norm_w per token
    // (cpu.go:81-98), the norm taken from the rows' sums of squares in dm.ssq; a RESID product also
    // writes its output rows' sums of squares there (with ssq_out set)
    const float *norm_w;
    bool ssq_out;
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
    const QMat &ma = mat_at(ga.a, seg);
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

// ------------------------------------------------ tensor-core products --
// The same products on the 5th-generation tensor cores (tcgen05), exact to
// float32 level by error-compensated splitting.  A CTA owns 128 weight rows x
// 64 tokens (the MMA's M x N) and a share of K (the cluster split and the
// distributed-shared-memory reduction of k_gemm).  Per 32-wide K block:
//   - the weights are dequantised exactly in float32 (d * (q - 8) of Q4_0 has
//     at most 15 significant bits, d * q of Q8_0 18; Q4_1's d * q + m is the
//     float32 result) and split into bf16 pieces a = a1 + a2 (+ a3), each the
//     bf16 rounding of what the earlier pieces leave: exact for Q4_0 with two
//     pieces, and to float32 with three;
//   - the activations are split the same way into three bf16 pieces
//     x = x1 + x2 + x3 (exact for every float32);
//   - tcgen05.mma (kind::f16, bf16 x bf16 -> f32 in tensor memory) adds the
//     piece products a1 x1, a1 x2, a2 x1, a1 x3, a2 x2 (and a3 x1): every
//     product of two bf16 pieces is exact, and the dropped ones are below
//     2^-24 of a x (|a2|, |x2| <= 2^-9, |a3|, |x3| <= 2^-17 relative).
// The operands are written by all threads into shared memory in the MMA's
// K-major canonical layout without swizzle (8-row x 16-byte core matrices),
// two stages deep, so one block's split overlaps the previous block's MMAs;
// one thread issues the MMAs and tcgen05.commit signals an mbarrier when they
// have read a stage.  The accumulator (128 lanes x 64 columns of f32 per
// matrix) is read back with tcgen05.ld and goes through k_gemm's epilogues.
namespace tc {

constexpr int kMR = 128;                   // weight rows per CTA (MMA M)
constexpr int kMN = 64;                    // tokens per CTA (MMA N; rows of X past m are zero)
constexpr int kAPiece = kMR * 32 * 2;      // one bf16 piece of a 128 x 32 weight block (8 KB)
constexpr int kBPiece = kMN * 32 * 2;      // one bf16 piece of a 64 x 32 activation block (4 KB)
constexpr int kPartLd = kMR + 4;           // floats per token of the accumulator copy in shared memory
constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s: the limit of a wait for the tensor cores

constexpr int kDepth = 4;                  // K blocks of raw operands in flight per staging thread (cp.async)
constexpr int kNwFloats = 1024;            // norm weights of the CTA's K range (a normed product has K = embd <= 1024)

// Shared memory: two stages of bf16 operands (the accumulators' copy for the
// epilogue aliases them), then kDepth stages of raw operands, then the norm
// weights, then the mbarriers.  A raw stage holds, per staging thread, the
// quant bytes (16 B) and the scale / minimum words (8 B) of its row share for
// each matrix, then its 32 activation bytes (two 16-byte halves).
__host__ __device__ constexpr int stage_bytes(int na) { return na * 3 * kAPiece + 3 * kBPiece; }
__host__ __device__ constexpr int raw_bytes(int na) { return na * kGT * 24 + kGT * 32; }
__host__ __device__ constexpr int raw_off(int na) { return 2 * stage_bytes(na); }
__host__ __device__ constexpr int nw_off(int na) { return raw_off(na) + kDepth * raw_bytes(na); }
__host__ __device__ constexpr int part_bytes(int na) { return na * kMN * kPartLd * 4; }
__host__ __device__ constexpr int smem_bytes(int na) {
    return (nw_off(na) + kNwFloats * 4 > part_bytes(na) ? nw_off(na) + kNwFloats * 4 : part_bytes(na)) + 64;
}
static_assert(smem_bytes(2) + 4096 <= 232448, "the products' shared memory exceeds the per-block maximum");

// Byte offset of element (row, k) of a K-major canonical operand with `groups`
// 8-row groups: core matrix (row / 8, k / 8) at ((k / 8) * groups + row / 8) * 128,
// rows 16 bytes apart inside it.  So the stride between 8-row groups (SBO) is
// 128 bytes and between 8-element K chunks (LBO) groups * 128.
__device__ __forceinline__ uint32_t cm_off(int row, int kc, int groups) {
    return (uint32_t)((kc * groups + (row >> 3)) * 128 + (row & 7) * 16);
}

// Shared-memory matrix descriptor (SWIZZLE_NONE, version 1 for sm_100).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor: kind::f16 with bf16 A and B, f32 D, both K-major, M = 128, N = 64.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kMN >> 3) << 17) |
                            ((uint32_t)(kMR >> 4) << 24);

__device__ __forceinline__ uint32_t su32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}

__device__ __forceinline__ bool bar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(su32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits (bounded) for phase `parity` of an mbarrier; false after the limit (or
// once another CTA has recorded an error).
__device__ __forceinline__ bool bar_wait(uint64_t *bar, uint32_t parity, int *err) {
    if (bar_try(bar, parity)) return true;
    const uint64_t t0 = gtime();
    unsigned spins = 0;
    while (!bar_try(bar, parity)) {
        if ((++spins & 63) == 0) {
            if (*(volatile int *)err) return false;
            if (gtime() - t0 > kWaitNs) {
                atomicExch(err, DEV_MMA_TIMEOUT);
                return false;
            }
        }
    }
    return true;
}

// Two floats into three bf16 pieces each (packed pairs, first value in the low half).
__device__ __forceinline__ void split3(float v0, float v1, uint32_t &p1, uint32_t &p2, uint32_t &p3) {
    const __nv_bfloat162 h1 = __floats2bfloat162_rn(v0, v1);
    const float2 f1 = __bfloat1622float2(h1);
    const float r0 = v0 - f1.x, r1 = v1 - f1.y;  // exact
    const __nv_bfloat162 h2 = __floats2bfloat162_rn(r0, r1);
    const float2 f2 = __bfloat1622float2(h2);
    const __nv_bfloat162 h3 = __floats2bfloat162_rn(r0 - f2.x, r1 - f2.y);
    p1 = *reinterpret_cast<const uint32_t *>(&h1);
    p2 = *reinterpret_cast<const uint32_t *>(&h2);
    p3 = *reinterpret_cast<const uint32_t *>(&h3);
}

// Eight values (one core-matrix row) split and stored into pieces 0..NP-1 (piece stride `pstride` bytes).
template <int NP>
__device__ __forceinline__ void store_split8(uint8_t *base, uint32_t off, int pstride, const float (&v)[8]) {
    uint32_t p[3][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (NP == 3) {
            split3(v[2 * i], v[2 * i + 1], p[0][i], p[1][i], p[2][i]);
        } else {
            const __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            const float2 f1 = __bfloat1622float2(h1);
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i] - f1.x, v[2 * i + 1] - f1.y);
            p[0][i] = *reinterpret_cast<const uint32_t *>(&h1);
            p[1][i] = *reinterpret_cast<const uint32_t *>(&h2);
        }
    }
#pragma unroll
    for (int j = 0; j < NP; ++j) *reinterpret_cast<uint4 *>(base + j * pstride + off) = make_uint4(p[j][0], p[j][1], p[j][2], p[j][3]);
}

// Staging thread t takes weight row t % 128, half t / 128 of each block, and
// token t % 64, columns 8 (t / 64)..+7 of the activations: consecutive
// threads then store consecutive 16-byte rows of a core matrix, which is free
// of shared-memory bank conflicts.
__device__ __forceinline__ int a_row() { return threadIdx.x & (kMR - 1); }
__device__ __forceinline__ int a_half() { return threadIdx.x >> 7; }
__device__ __forceinline__ int b_tok() { return threadIdx.x & (kMN - 1); }
__device__ __forceinline__ int b_col8() { return threadIdx.x >> 6; }

// A thread's raw share of one weight block: row a_row(), half a_half() of its
// quants (Q4: bytes 8h..8h+7; Q8_0: bytes 16h..16h+15), its scale and (Q4_1)
// minimum.
struct ARaw {
    uint4 w;
    float d, mn;
    int type;  // 0: no row (past the matrices)
};

// Where a thread's raw share of block kb of one matrix lives: the quant bytes
// at q + kb * qstep, and the 4-byte word holding the scales of its row pair at
// d + kb * 16 (its own in the high half when hi), the minima mstep bytes after.
// The thread's row is the same for every block, so this is set up once.
struct ASrc {
    const uint8_t *q, *d;
    int type, hi, qstep, mstep;
};

__device__ __forceinline__ void a_src(const MatSet &ms, int total, int r0, ASrc &s) {
    const int row = a_row(), h = a_half();
    s.q = s.d = nullptr;
    s.type = s.hi = s.qstep = s.mstep = 0;
    if (r0 + row >= total) return;
    int lr = 0;
    const QMat &m = mat_at(ms, mat_of(ms, r0 + row, lr));
    const uint8_t *tile = m.tiles + (size_t)(lr >> 3) * m.tile_bytes;
    const int r = lr & 7;
    const bool q8 = m.type == 8;
    s.type = m.type;
    s.hi = r & 1;
    s.qstep = q8 ? 256 : 128;
    s.q = tile + r * (q8 ? 32 : 16) + h * (q8 ? 16 : 8);
    s.d = tile + (size_t)m.nb * s.qstep + (r & ~1) * 2;
    s.mstep = m.nb * 16;
}

__device__ __forceinline__ void cp4(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp8(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
// 16 bytes, of which the first n (0 or 16) are read and the rest zero-filled
__device__ __forceinline__ void cp16(uint32_t dst, const void *src, uint32_t n = 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// This thread's raw weight shares (as[j]) of block kb into the raw stage at
// shared address raw.  The weights are constant, so these copies may precede
// the wait for the previous kernel.
template <int NM>
__device__ __forceinline__ void copy_raw_a(const ASrc (&as)[NM], int kb, uint32_t raw) {
    const int t = threadIdx.x;
#pragma unroll
    for (int j = 0; j < NM; ++j) {
        const ASrc &s = as[j];
        if (!s.type) continue;
        const uint32_t aq = raw + (j * kGT + t) * 16, ad = raw + NM * kGT * 16 + (j * kGT + t) * 8;
        const uint8_t *q = s.q + (size_t)kb * s.qstep, *d = s.d + (size_t)kb * 16;
        if (s.type == 8) cp16(aq, q);
        else cp8(aq, q);
        cp4(ad, d);
        if (s.type == 3) cp4(ad + 4, d + s.mstep);
    }
}

// This thread's 8 activations of block kb (token b_tok(), columns 8 b_col8()..+7;
// zeros for tokens past m) into the raw stage at shared address raw.
template <int NM>
__device__ __forceinline__ void copy_raw_b(const float *x, int K, int m, int kb, uint32_t raw) {
    const int tok = b_tok(), c = b_col8();
    const bool v = tok < m;
    const float *p = v ? x + (size_t)tok * K + kb * 32 + 8 * c : x;
    const uint32_t bx = raw + NM * kGT * 24 + threadIdx.x * 16;
    cp16(bx, p, v ? 16u : 0u);
    cp16(bx + kGT * 16, p + 4, v ? 16u : 0u);
}

// Programmatic dependent launch: wait until the grids this one depends on
// have completed and their writes are visible (a no-op without such a
// dependency), and allow the dependent grid to launch.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The raw share of matrix j in a raw stage, as an ARaw.
template <int NM>
__device__ __forceinline__ ARaw raw_a(const ASrc &s, const uint8_t *raw, int j) {
    ARaw R;
    R.type = s.type;
    R.d = R.mn = 0.f;
    R.w = make_uint4(0u, 0u, 0u, 0u);
    if (!s.type) return R;
    const int t = threadIdx.x;
    R.w = *reinterpret_cast<const uint4 *>(raw + (j * kGT + t) * 16);
    const uint2 dw = *reinterpret_cast<const uint2 *>(raw + NM * kGT * 16 + (j * kGT + t) * 8);
    R.d = __half2float(__ushort_as_half((unsigned short)(s.hi ? dw.x >> 16 : dw.x & 0xFFFFu)));
    if (s.type == 3) R.mn = __half2float(__ushort_as_half((unsigned short)(s.hi ? dw.y >> 16 : dw.y & 0xFFFFu)));
    return R;
}

// The raw share dequantised exactly in float32 and split into the NP bf16
// pieces of the A operand at a (Q4: elements 8h.. -> chunk h and 16+8h.. ->
// chunk 2+h; Q8_0: 16h.. -> chunk 2h and 16h+8.. -> chunk 2h+1).  A missing
// row is zero.
template <int NP>
__device__ __forceinline__ void stage_a(const ARaw &R, uint8_t *a) {
    const int row = a_row(), h = a_half();
    float lo[8], hi[8];
    if (R.type == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) lo[i] = hi[i] = 0.f;
    } else if (R.type == 8) {
        const uint32_t u[4] = {R.w.x ^ 0x80808080u, R.w.y ^ 0x80808080u, R.w.z ^ 0x80808080u, R.w.w ^ 0x80808080u};
        constexpr float off = 8388736.f;  // 2^23 + 128
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = R.d * (b2f(u[0], i) - off), lo[4 + i] = R.d * (b2f(u[1], i) - off);
            hi[i] = R.d * (b2f(u[2], i) - off), hi[4 + i] = R.d * (b2f(u[3], i) - off);
        }
    } else {
        const uint32_t l0 = R.w.x & 0x0F0F0F0Fu, l1 = R.w.y & 0x0F0F0F0Fu;
        const uint32_t h0 = (R.w.x >> 4) & 0x0F0F0F0Fu, h1 = (R.w.y >> 4) & 0x0F0F0F0Fu;
        if (R.type == 3) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lo[i] = fmaf(R.d, b2f(l0, i) - 8388608.f, R.mn), lo[4 + i] = fmaf(R.d, b2f(l1, i) - 8388608.f, R.mn);
                hi[i] = fmaf(R.d, b2f(h0, i) - 8388608.f, R.mn), hi[4 + i] = fmaf(R.d, b2f(h1, i) - 8388608.f, R.mn);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lo[i] = R.d * (b2f(l0, i) - 8388616.f), lo[4 + i] = R.d * (b2f(l1, i) - 8388616.f);
                hi[i] = R.d * (b2f(h0, i) - 8388616.f), hi[4 + i] = R.d * (b2f(h1, i) - 8388616.f);
            }
        }
    }
    const bool q8 = R.type == 8;
    store_split8<NP>(a, cm_off(row, q8 ? 2 * h : h, kMR / 8), kAPiece, lo);
    store_split8<NP>(a, cm_off(row, q8 ? 2 * h + 1 : 2 + h, kMR / 8), kAPiece, hi);
}

// The block into the three B pieces; with a norm, each value is (x * s) * w
// first (cpu.go:94-97's rounding points), s the token's 1 / rms.
__device__ __forceinline__ void stage_b(const float4 (&u)[4], bool norm, float s, uint8_t *b) {
    const int tok = b_tok(), c = b_col8();
    float v[8] = {u[0].x, u[0].y, u[0].z, u[0].w, u[1].x, u[1].y, u[1].z, u[1].w};
    if (norm) {
        const float w[8] = {u[2].x, u[2].y, u[2].z, u[2].w, u[3].x, u[3].y, u[3].z, u[3].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], s), w[i]);
    }
    store_split8<3>(b, cm_off(tok, c, kMN / 8), kBPiece, v);
}

#define TC_LD32(taddr, r)                                                                                          \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, " \
                 "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, " \
                 "[%32];"                                                                                          \
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), \
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),       \
                   "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),     \
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),     \
                   "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                                                          \
                 : "r"(taddr))

}  // namespace tc

// The tensor-core products' epilogue, split in two: epi_in gathers an item's
// inputs that do not depend on the product (destination, QKV bias and RoPE
// (cos, sin), the residual's old values), so that a CTA can load them while
// its MMAs finish and its cluster meets; epi_out applies them to the item's
// 4 summed rows, as epilogue() does.
struct EpiIn {
    float *dst;    // the item's first output element
    float a[4];    // QKV: the bias; RESID: the residual rows' old values
    float2 cs[2];  // QKV: (cos, sin) of the item's two rotary pairs
    int n;         // outputs of the item (0: none)
    bool hasb, rot;
};

template <int EPI>
__device__ __forceinline__ EpiIn epi_in(const GemmArgs &ga, const DevModel &dm, int g, int t, int total) {
    EpiIn e;
    e.dst = nullptr;
    e.n = 0;
    e.hasb = e.rot = false;
#pragma unroll
    for (int c = 0; c < 4; ++c) e.a[c] = 0.f;
    e.cs[0] = e.cs[1] = make_float2(0.f, 0.f);
    if (t >= ga.m || g >= total) return e;
    int la = 0;
    const int seg = mat_of(ga.a, g, la);
    const QMat &ma = mat_at(ga.a, seg);
    if constexpr (EPI == EPI_RESID) {
        e.n = min(4, ma.rows - la);
        e.dst = ga.out + (size_t)t * ga.out_ld + g;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (c < e.n) e.a[c] = __ldcg(e.dst + c);
    } else if constexpr (EPI == EPI_SWIGLU) {
        e.n = max(0, min(4, min(dm.ff, ma.rows) - g));
        e.dst = ga.out + (size_t)t * ga.out_ld + g;
    } else if constexpr (EPI == EPI_QKV) {  // kernels_fused.go:212-224; cpu.go:279-303
        const int pos = ga.tb ? ga.tb->pos[t] : (int)dm.state[0] + t;
        const Layer &L = dm.layer[ga.l];
        const float *bias = seg == 0 ? L.bq : seg == 1 ? L.bk : L.bv;
        e.hasb = bias != nullptr;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (bias) e.a[c] = __ldg(bias + la + c);
        e.rot = seg < 2;
        if (seg < 2) {
            const int hp = dm.head_dim >> 1;
#pragma unroll
            for (int c = 0; c < 4; c += 2)
                e.cs[c >> 1] = __ldg(reinterpret_cast<const float2 *>(dm.rope_cs) + (size_t)pos * hp +
                                     (((la + c) % dm.head_dim) >> 1));
        }
        float *kv = ga.tb ? ga.tb->kv + ((size_t)ga.tb->slot[t] * ga.tb->layers + ga.l) * 2 * (size_t)dm.ctx * dm.kvd
                          : L.kv;
        e.dst = seg == 0 ? dm.q + (size_t)t * dm.embd + la
                         : kv + ((seg == 1 ? 0 : (size_t)dm.ctx) + pos) * (size_t)dm.kvd + la;
        e.n = 4;
    }
    return e;
}

// Applies an item's inputs to its summed rows v; returns the sum of squares of a residual's new values.
template <int EPI, int NM>
__device__ __forceinline__ float epi_out(const EpiIn &e, const float (&v)[NM][4]) {
    float sq = 0.f;
    if constexpr (EPI == EPI_RESID) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (c < e.n) {
                const float nv = __fadd_rn(e.a[c], v[0][c]);
                e.dst[c] = nv;
                sq = fmaf(nv, nv, sq);
            }
    } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (c < e.n) {
                const float g = v[0][c], u = v[NM - 1][c];
                const float den = __fadd_rn(1.f, (float)exp(-(double)g));  // cpu.go:345
                e.dst[c] = __fmul_rn(__fdiv_rn(g, den), u);
            }
    } else if constexpr (EPI == EPI_QKV) {
        if (e.n) {
            float o[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) o[c] = e.hasb ? __fadd_rn(v[0][c], e.a[c]) : v[0][c];
            if (e.rot) {  // rotate adjacent pairs (cpu.go:371-385)
#pragma unroll
                for (int c = 0; c < 4; c += 2) {
                    const float2 cs = e.cs[c >> 1];
                    const float x0 = o[c], x1 = o[c + 1];
                    o[c] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
                    o[c + 1] = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) e.dst[c] = o[c];
        }
    }
    return sq;
}

// grid (row tiles of 128, splits), cluster (1, splits, 1); 9 warps.  NM
// matrices (2: gate and up) share the activations; each has its own
// accumulator (64 tensor-memory columns).  Warps 0-7 stage the operands of
// each K block (two stages deep) and signal `full`; warp 8 allocates the
// tensor memory, waits for `full`, issues the block's MMAs from one thread
// and commits them to `empty`, which releases the stage.  No block-wide
// barrier separates K blocks, so staging overlaps the tensor cores.
constexpr int kMT = kGT + 32;  // threads of k_mma: 8 staging warps and the MMA warp
constexpr int kMaxSplit = 16;  // CTAs of a cluster along K

template <int EPI>
__global__ void __launch_bounds__(kMT, 1) k_mma(const __grid_constant__ GemmArgs ga) {
    using namespace tc;
    constexpr int NM = EPI == EPI_SWIGLU ? 2 : 1;
    constexpr int kCols = 64 * NM;  // tensor-memory columns (a power of 2, >= 32)
    extern __shared__ __align__(1024) uint8_t tsm[];
    __shared__ uint32_t tmem_slot;
    uint64_t *full = reinterpret_cast<uint64_t *>(tsm + smem_bytes(NM) - 64);  // [2]: a stage is staged
    uint64_t *empty = full + 2;                                                // [2]: its MMAs have read it
    const DevModel &dm = *ga.dm;
    const int rt = blockIdx.x, sp = blockIdx.y, r0 = rt * kMR;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool mma_warp = warp == kGT / 32;
    const int kb0 = ga.nb * sp / ga.splits, kb1 = ga.nb * (sp + 1) / ga.splits;
    const int K = ga.nb * 32, nblk = kb1 - kb0;
    // bf16 pieces of the weights: two when every matrix is Q4_0 (exact), else three
    int np = 2;
    for (int i = 0; i < ga.a.nm; ++i) np = ga.a.m[i].type != 2 ? 3 : np;
    for (int i = 0; i < (NM == 2 ? ga.b.nm : 0); ++i) np = ga.b.m[i].type != 2 ? 3 : np;
    if (mma_warp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_slot)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __shared__ float s_norm[kMN];
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(full + i)), "r"(kGT / 32));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(empty + i)));
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;
    bool ok = true;
    // epilogue work items, token-major (t = it / 32, u = it % 32), CTA sp taking a contiguous share, so that
    // a warp's threads cover consecutive 4-row groups of one token (coalesced epilogue stores).  With
    // ssq_out (a residual product) CTA sp takes whole tokens, a warp per token, so that the warp can sum
    // the squares of its token's new rows.
    const int S = ga.splits;
    const bool tok_rows = EPI == EPI_RESID && ga.ssq_out;
    const int items = (kMR / 4) * ga.m;
    const int i0 = tok_rows ? 32 * (ga.m * sp / S) : items * sp / S;
    const int i1 = tok_rows ? 32 * (ga.m * (sp + 1) / S) : items * (sp + 1) / S;
    int total = 0;
    for (int i = 0; i < ga.a.nm; ++i) total += ga.a.m[i].rows;
    EpiIn pre;  // the inputs of this thread's first item, loaded once its operands are staged
    pre.n = 0;
    if (!mma_warp) {
        int tot[2] = {0, 0};
        for (int i = 0; i < ga.a.nm; ++i) tot[0] += ga.a.m[i].rows;
        for (int i = 0; i < (NM == 2 ? ga.b.nm : 0); ++i) tot[1] += ga.b.m[i].rows;
        // Raw operands travel by cp.async kDepth - 1 blocks ahead of their staging; each thread copies the
        // raw bytes it dequantises itself, so its own cp.async group waits are all the ordering needed.
        // The constant operands of the first blocks (weights, norm weights) are requested before the wait
        // for the previous kernel, whose outputs (activations, sums of squares) are read after it.
        // Groups: {weights of blocks 0..kDepth-2, norm weights, activations of block 0}, then the
        // activations of blocks 1..kDepth-2, then {weights, activations} of each later block.
        const bool norm = ga.norm_w != nullptr;
        const int ntiles = (ga.nb * 32 + kMR - 1) / kMR;
        ASrc as[NM];
        for (int j = 0; j < NM; ++j) a_src(j == 0 ? ga.a : ga.b, tot[j], r0, as[j]);
        const float *s_nw = reinterpret_cast<const float *>(tsm + nw_off(NM));
        const uint32_t raw0 = su32(tsm + raw_off(NM));
#pragma unroll
        for (int p = 0; p < kDepth - 1; ++p)
            if (p < nblk) copy_raw_a<NM>(as, kb0 + p, raw0 + p * raw_bytes(NM));
        if (norm)  // the norm weights of the CTA's K range
            for (int i = threadIdx.x; i < nblk * 8; i += kGT) cp16(su32(s_nw) + i * 16, ga.norm_w + kb0 * 32 + i * 4);
        griddep_wait();
        // RMSNorm inputs: each token's sums of squares per 128-row tile
        float ssv[kSsqTiles];
#pragma unroll
        for (int i = 0; i < kSsqTiles; ++i)
            ssv[i] = norm && (int)threadIdx.x < ga.m && i < ntiles ? __ldcg(dm.ssq + (size_t)threadIdx.x * kSsqTiles + i)
                                                                    : 0.f;
#pragma unroll
        for (int p = 0; p < kDepth - 1; ++p) {
            if (p < nblk) copy_raw_b<NM>(ga.x, K, ga.m, kb0 + p, raw0 + p * raw_bytes(NM));
            cp_commit();
        }
        // RMSNorm scale of each token (cpu.go:81-98: 1 / sqrt(mean of squares + eps) in double, rounded
        // to float), from the row's sums of squares per 128-row tile, added in tile order, then shared by
        // the staging warps with the norm weights (named barrier 1)
        float sn = 1.f;
        if (norm) {
            if ((int)threadIdx.x < ga.m) {
                float ss = 0.f;
#pragma unroll
                for (int i = 0; i < kSsqTiles; ++i)
                    if (i < ntiles) ss += ssv[i];
                s_norm[threadIdx.x] = (float)(1.0 / sqrt((double)__fadd_rn(__fdiv_rn(ss, (float)(ga.nb * 32)), dm.eps)));
            }
            cp_wait<kDepth - 2>();  // this thread's norm-weight copies (the oldest group) have landed
            asm volatile("bar.sync 1, %0;" ::"n"(kGT) : "memory");
            if (b_tok() < ga.m) sn = s_norm[b_tok()];
        }
        const int c8 = 8 * b_col8();
        for (int i = 0; i < nblk; ++i) {
            const int pf = i + kDepth - 1;
            if (pf < nblk) {
                copy_raw_a<NM>(as, kb0 + pf, raw0 + (pf % kDepth) * raw_bytes(NM));
                copy_raw_b<NM>(ga.x, K, ga.m, kb0 + pf, raw0 + (pf % kDepth) * raw_bytes(NM));
            }
            cp_commit();
            cp_wait<kDepth - 1>();  // block i's raw operands (this thread's copies) have landed
            const int st = i & 1;
            uint8_t *stage = tsm + st * stage_bytes(NM);
            if (i >= 2) {  // the MMAs of block i - 2 have read this stage (one wait per warp)
                bool w = true;
                if (lane == 0) w = bar_wait(empty + st, ((i >> 1) - 1) & 1, dm.err);
                if (!__shfl_sync(kFull, w, 0)) {
                    ok = false;
                    break;
                }
            }
            const uint8_t *raw = tsm + raw_off(NM) + (i % kDepth) * raw_bytes(NM);
            for (int j = 0; j < NM; ++j) {
                const ARaw R = raw_a<NM>(as[j], raw, j);
                if (np == 3) stage_a<3>(R, stage + j * 3 * kAPiece);
                else stage_a<2>(R, stage + j * 3 * kAPiece);
            }
            float4 xb[4];
            const uint8_t *bx = raw + NM * kGT * 24 + threadIdx.x * 16;
            xb[0] = *reinterpret_cast<const float4 *>(bx);
            xb[1] = *reinterpret_cast<const float4 *>(bx + kGT * 16);
            if (norm) {
                const float4 *w4 = reinterpret_cast<const float4 *>(s_nw + (size_t)i * 32 + c8);
                xb[2] = w4[0], xb[3] = w4[1];
            }
            stage_b(xb, norm, sn, stage + NM * 3 * kAPiece);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the operands, to the tensor cores' proxy
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(full + st)) : "memory");
        }
        cp_wait<0>();  // nothing left in flight (the error path leaves copies behind)
        if constexpr (EPI != EPI_ARGMAX) {
            const int it = i0 + (int)threadIdx.x;
            if (it < i1) pre = epi_in<EPI>(ga, dm, r0 + 4 * (it & 31), it >> 5, total);
        }
    } else if (lane == 0) {
        // descriptors of stage 0, piece 0, K step 0 (the others are byte offsets added to the address field)
        const uint64_t da0 = sdesc(su32(tsm), (kMR / 8) * 128, 128);
        const uint64_t db0 = sdesc(su32(tsm + NM * 3 * kAPiece), (kMN / 8) * 128, 128);
        constexpr uint64_t pa[6] = {0, 0, 1, 0, 1, 2}, pb[6] = {0, 1, 0, 2, 1, 0};  // exact products down to 2^-18 of a x
        const int npairs = np == 3 ? 6 : 5;
        for (int i = 0; i < nblk; ++i) {
            const int st = i & 1;
            if (!bar_wait(full + st, (i >> 1) & 1, dm.err)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint64_t so = (uint64_t)(st * stage_bytes(NM)) >> 4;
            for (int j = 0; j < NM; ++j)
#pragma unroll
                for (int ks = 0; ks < 2; ++ks)
#pragma unroll
                    for (int q = 0; q < 6; ++q) {
                        if (q >= npairs) break;
                        const uint64_t da =
                            da0 + so + (((uint64_t)j * 3 * kAPiece + pa[q] * kAPiece + ks * 2 * (kMR / 8) * 128) >> 4);
                        const uint64_t db = db0 + so + ((pb[q] * kBPiece + ks * 2 * (kMN / 8) * 128) >> 4);
                        mma(tmem + j * 64, da, db, (i > 0 || ks > 0 || q > 0) ? 1u : 0u);
                    }
            commit(empty + st);
        }
    }
    // the last block's MMAs (and so all before them) are done
    if (ok && nblk > 0 && !mma_warp) {
        bool w = true;
        if (lane == 0) w = bar_wait(empty + ((nblk - 1) & 1), ((nblk - 1) >> 1) & 1, dm.err);
        ok = __shfl_sync(kFull, w, 0);
    }
    ok = !__syncthreads_or(!ok);
    griddep_launch();  // the next kernel may start its own set-up while this one reduces and stores
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // accumulators -> part[j][token][row] (token-major, so that 4 consecutive rows of a token are one float4;
    // the stages are free): warp w < 8 reads lanes 32 (w % 4).. of columns 32 (w / 4)..
    float *part = reinterpret_cast<float *>(tsm);
    if (ok && !mma_warp) {
        const int row = 32 * (warp & 3) + lane, c0 = 32 * (warp >> 2);
        for (int j = 0; j < NM; ++j) {
            uint32_t r[32];
            if (nblk > 0) {
                TC_LD32(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + j * 64 + c0, r);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) r[c] = 0u;
            }
            float *pr = part + ((size_t)j * kMN + c0) * kPartLd + row;
#pragma unroll
            for (int c = 0; c < 32; ++c) pr[c * kPartLd] = __uint_as_float(r[c]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (mma_warp) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
    if (EPI == EPI_ARGMAX) {  // no split: the tile's best row per token
        __shared__ float bvs[4][kMN];
        __shared__ int bis[4][kMN];
        if (!mma_warp) {
            const int t = threadIdx.x & 63, seg = threadIdx.x >> 6;
            float bv = -FLT_MAX;
            int bi = 0x7fffffff;
            for (int rr = seg * 32; ok && rr < seg * 32 + 32; ++rr) {
                const int row = r0 + rr;
                const float v = part[(size_t)t * kPartLd + rr];
                if (row < dm.vocab && better(v, row, bv, bi)) bv = v, bi = row;
            }
            bvs[seg][t] = bv, bis[seg][t] = bi;
        }
        __syncthreads();
        if (ok && threadIdx.x < ga.m) {
            float v = bvs[0][threadIdx.x];
            int ix = bis[0][threadIdx.x];
            for (int q = 1; q < 4; ++q)
                if (better(bvs[q][threadIdx.x], bis[q][threadIdx.x], v, ix)) v = bvs[q][threadIdx.x], ix = bis[q][threadIdx.x];
            dm.gam[(size_t)threadIdx.x * gridDim.x + rt] = make_float2(v, __int_as_float(ix));
        }
    } else {
        // the cluster's partials summed in rank order, then the epilogue: work item (4-row group u, token t)
        cg::cluster_group cl = cg::this_cluster();
        if (ga.splits > 1) cl.sync();
        // (with tok_rows i0 is a multiple of 32, so every warp's 32 items are one token's)
        for (int it = i0 + (int)threadIdx.x; ok && !mma_warp && it < i1; it += kGT) {
            const int t = it >> 5, u = it & 31;
            const int g = r0 + 4 * u;
            const EpiIn e = it == i0 + (int)threadIdx.x ? pre : epi_in<EPI>(ga, dm, g, t, total);
            float sq = 0.f;
            if (g < total) {
                // the ranks' float4s of rows 4u..4u+3 at token t, loaded 8 ranks at a time, summed in rank order
                float v[NM][4];
#pragma unroll
                for (int j = 0; j < NM; ++j) v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.f;
#pragma unroll
                for (int r0 = 0; r0 < kMaxSplit; r0 += 8) {
                    if (r0 >= S) break;
                    float4 pv[8][NM];
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        if (r0 + r < S) {
                            const float *rs = S > 1 ? cl.map_shared_rank(part, r0 + r) : part;
#pragma unroll
                            for (int j = 0; j < NM; ++j)
                                pv[r][j] = *reinterpret_cast<const float4 *>(rs + ((size_t)j * kMN + t) * kPartLd + 4 * u);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < NM; ++j)
#pragma unroll
                        for (int r = 0; r < 8; ++r)
                            if (r0 + r < S)
                                v[j][0] += pv[r][j].x, v[j][1] += pv[r][j].y, v[j][2] += pv[r][j].z, v[j][3] += pv[r][j].w;
                }
                sq = epi_out<EPI, NM>(e, v);
            }
            if (tok_rows) {
                // a warp per token: every lane takes part in the sum (rows past the matrix add 0)
#pragma unroll
                for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(kFull, sq, o);
                if (u == 0) dm.ssq[(size_t)t * kSsqTiles + rt] = sq;
            }
        }
        if (ga.splits > 1) cl.sync();  // the partials stay readable until every CTA of the cluster is done
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

// Clusters of s CTAs (s = 1..16) of each tensor-core product kernel that are
// resident at once, by device (cudaOccupancyMaxActiveClusters: one CTA per
// SM, and a cluster's CTAs in one GPC), measured by prepare_products.
constexpr int kMaxDevices = 64;
int g_mma_clusters[kMaxDevices][4][kMaxSplit + 1];

// CTAs along K per row tile for the tensor-core products.  Every cluster must
// be resident at once (a second wave would double the time) and each CTA
// must get at least 2 K blocks; among those splits, the one whose CTAs take
// the fewest K blocks at most (the cluster waits for its slowest CTA), and
// of equals the smallest (less to reduce).  Sizes above 8 are non-portable:
// a GPC holds one such cluster at most.
int mma_splits(int epi, int row_tiles, int nb) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
    int best = 1, most = nb;
    for (int s = 2; s <= kMaxSplit; ++s)
        if (nb >= 2 * s && row_tiles <= g_mma_clusters[dev][epi][s] && (nb + s - 1) / s < most)
            best = s, most = (nb + s - 1) / s;
    return best;
}

template <int EPI>
cudaError_t mma_gemm(const GemmArgs &base, int rows, int nsm, cudaStream_t st, bool pdl) {
    constexpr int NM = EPI == EPI_SWIGLU ? 2 : 1;
    GemmArgs ga = base;
    const int row_tiles = (rows + tc::kMR - 1) / tc::kMR;
    ga.splits = EPI == EPI_ARGMAX ? 1 : mma_splits(EPI, row_tiles, ga.nb);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(row_tiles, ga.splits);
    cfg.blockDim = dim3(kMT);
    cfg.dynamicSmemBytes = tc::smem_bytes(NM);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = ga.splits, attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, k_mma<EPI>, ga);
}

template <int EPI>
cudaError_t product(bool tensor, const GemmArgs &ga, int rows, int nsm, cudaStream_t st, bool pdl = false) {
    return tensor ? mma_gemm<EPI>(ga, rows, nsm, st, pdl) : gemm<EPI>(ga, rows, nsm, st);
}

}  // namespace

cudaError_t prepare_products() {
    const std::pair<const void *, int> fs[] = {{(const void *)k_mma<EPI_QKV>, tc::smem_bytes(1)},
                                               {(const void *)k_mma<EPI_RESID>, tc::smem_bytes(1)},
                                               {(const void *)k_mma<EPI_SWIGLU>, tc::smem_bytes(2)},
                                               {(const void *)k_mma<EPI_ARGMAX>, tc::smem_bytes(1)}};
    for (const auto &f : fs) {
        cudaError_t e = cudaFuncSetAttribute(f.first, cudaFuncAttributeMaxDynamicSharedMemorySize, f.second);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f.first, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    for (int k = 0; k < 4; ++k)
        for (int s = 1; s <= kMaxSplit; ++s) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(1, s);
            cfg.blockDim = dim3(kMT);
            cfg.dynamicSmemBytes = fs[k].second;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = s, attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            e = cudaOccupancyMaxActiveClusters(&n, fs[k].first, &cfg);
            if (e != cudaSuccess) {
                if (s <= 8) return e;
                cudaGetLastError();  // a device without clusters of 16: that split is not used
                n = 0;
            }
            g_mma_clusters[dev][k][s] = n;
        }
    return cudaSuccess;
}

cudaError_t launch_layer_mm(const DevModel *dm, const DevModel &hd, const Shapes &s, int l, int m, int nsm,
                            cudaStream_t st, const TokBatch *tb, bool tensor) {
    const Layer &L = hd.layer[l];
    const int E = s.embd, F = s.ff;
    GemmArgs ga{};
    ga.dm = dm, ga.tb = tb, ga.m = m, ga.l = l;
    // QKV (the tensor-core products fold the RMSNorm in; the float32 ones read the normed rows)
    if (tensor) {
        ga.x = hd.x, ga.norm_w = L.attn_norm;
    } else {
        k_norm_rows<<<m, kGT, 0, st>>>(dm, L.attn_norm, nullptr, 0);
        ga.x = hd.h;
    }
    ga.nb = E / 32, ga.a = mats({&L.q, &L.k, &L.v});
    // (with the tensor-core products, every launch of the layer starts as a programmatic dependent of the
    // kernel before it, which lets it in once all of its CTAs have started or finished their main work)
    cudaError_t e = product<EPI_QKV>(tensor, ga, L.q.rows + L.k.rows + L.v.rows, nsm, st, tensor);
    ga.norm_w = nullptr;
    // attention (per token, per head and chunk of 64 positions)
    if (e == cudaSuccess) e = launch_attention(dm, s, l, m, st, tb, tensor);
    // x += Wo att
    ga.x = hd.att, ga.nb = E / 32, ga.a = mats({&L.o}), ga.out = hd.x, ga.out_ld = E, ga.ssq_out = tensor;
    if (e == cudaSuccess) e = product<EPI_RESID>(tensor, ga, L.o.rows, nsm, st, tensor);
    // act = SwiGLU(Wgate h, Wup h)
    if (tensor) {
        ga.x = hd.x, ga.norm_w = L.ffn_norm;
    } else {
        k_norm_rows<<<m, kGT, 0, st>>>(dm, L.ffn_norm, nullptr, 0);
        ga.x = hd.h;
    }
    ga.nb = E / 32, ga.a = mats({&L.gate}), ga.b = mats({&L.up}), ga.out = hd.act, ga.out_ld = F;
    if (e == cudaSuccess) e = product<EPI_SWIGLU>(tensor, ga, L.gate.rows, nsm, st, tensor);
    ga.norm_w = nullptr;
    // x += Wdown act
    ga.x = hd.act, ga.nb = F / 32, ga.a = mats({&L.down}), ga.b = MatSet{}, ga.out = hd.x, ga.out_ld = E;
    if (e == cudaSuccess) e = product<EPI_RESID>(tensor, ga, L.down.rows, nsm, st, tensor);
    return e;
}

cudaError_t launch_head_mm(const DevModel *dm, const DevModel &hd, const Shapes &s, TokBatch *tb, const int *rows_dev,
                           int rows, int nsm, cudaStream_t st, bool tensor) {
    k_norm_rows<<<rows, kGT, 0, st>>>(dm, hd.out_norm, rows_dev, 0);
    GemmArgs ga{};
    ga.dm = dm, ga.tb = tb, ga.m = rows, ga.x = hd.h, ga.nb = s.embd / 32, ga.a = mats({&hd.head});
    const cudaError_t e = product<EPI_ARGMAX>(tensor, ga, hd.head.rows, nsm, st);
    const int tile_rows = tensor ? tc::kMR : kTR;
    k_argmax_rows<<<rows, kGT, 0, st>>>(dm, tb, (hd.head.rows + tile_rows - 1) / tile_rows);
    return e;
}


}  // namespace llmb
