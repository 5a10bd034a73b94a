// Forward-pass kernels for sm_100a: batch-1 decode and chunked prefill of
// llama / qwen2 models with Q4_0, Q4_1 and Q8_0 weights and an f32 KV cache.
//
// The math restates the reference's CPU f32 path (cpu.go:225-366) and its
// fused WGSL kernels (kernels_fused.go:28-170, kernels.go:19-415); the
// shapes are B200's, not WebGPU's:
//   - a warp computes one tile of 8 output rows; lane (r, q) = (lane/4,
//     lane%4) owns row r and 8 of each block's 32 weights, so every block of
//     a tile is one 128- or 256-byte coalesced load and the 4 partial sums of
//     a row meet in two shuffles;
//   - nibbles become floats exactly with a byte permute into the mantissa of
//     2^23 (no integer-to-float conversion);
//   - RMSNorm is recomputed by every CTA that needs it (K1, K4 of
//     kernels_fused.go), RoPE and the KV append are the epilogue of the QKV
//     product, SwiGLU the epilogue of gate/up, the residual add the epilogue
//     of the output and down products;
//   - attention is split over chunks of 64 positions (flash-decoding, as K2
//     of kernels_fused.go:75-146); the last CTA of a head to finish merges
//     its chunks (K3's merge, kernels_fused.go:148-170), so the output
//     projection reads a finished vector;
//   - the vocab argmax (first index of the largest logit, cpu.go:387-397)
//     is fused into the head product: per-CTA partials, then a final pass.
// Every phase is a device function over work items; these kernels run m
// tokens per launch (prefill chunks, and decode with decode_mode 1).  The
// persistent decode kernel is in decode.cu.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>
#include <mutex>

#include "kernels.hpp"

namespace llmb {

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// 16 bytes global -> shared, asynchronously (both 16-byte aligned); completed by cp.async.wait_all.
__device__ __forceinline__ void cp_async16(float *dst, const float *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// Block-wide reductions over kThreads threads; red holds >= kWarps floats.
__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    return warp_sum(l < kWarps ? red[l] : 0.f);
}

// Byte k of v (0..255) plus 2^23, as a float: exact, one byte permute.
__device__ __forceinline__ float b2f(uint32_t v, int k) {
    return __int_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | k));
}

// ---------------------------------------------------------------- dot --
// Each returns, in all 4 lanes of row r = lane / 4, the dot product of tile
// row r with the vector xs (shared memory, nb * 32 floats).  A block's 8-term
// sum is f32; the sum over blocks is double, rounded once at the end.

// Q4_0: value d * (q - 8); byte j of a block holds element j (low nibble)
// and j + 16 (high nibble) (cpu.go:164-179).  Lane q owns bytes 4q..4q+3.
__device__ __forceinline__ float dot_q4_0(const uint8_t *__restrict__ tile, int nb, const float *__restrict__ xs,
                                          int lane) {
    const int r = lane >> 2, q = lane & 3;
    const uint32_t *qw = reinterpret_cast<const uint32_t *>(tile) + r * 4 + q;
    const __half *dp = reinterpret_cast<const __half *>(tile + (size_t)nb * 128) + r;
    const float *xp = xs + 4 * q;
    constexpr float kOff = 8388616.f;  // 2^23 + 8
    double acc = 0.0;
#pragma unroll 2
    for (int b = 0; b < nb; ++b) {
        const uint32_t w = __ldg(qw + b * 32);
        const float d = __half2float(__ldg(dp + b * 8));
        const float4 x0 = *reinterpret_cast<const float4 *>(xp + b * 32);
        const float4 x1 = *reinterpret_cast<const float4 *>(xp + b * 32 + 16);
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        float s = (b2f(lo, 0) - kOff) * x0.x;
        s = fmaf(b2f(hi, 0) - kOff, x1.x, s);
        s = fmaf(b2f(lo, 1) - kOff, x0.y, s);
        s = fmaf(b2f(hi, 1) - kOff, x1.y, s);
        s = fmaf(b2f(lo, 2) - kOff, x0.z, s);
        s = fmaf(b2f(hi, 2) - kOff, x1.z, s);
        s = fmaf(b2f(lo, 3) - kOff, x0.w, s);
        s = fmaf(b2f(hi, 3) - kOff, x1.w, s);
        acc = fma((double)d, (double)s, acc);
    }
    acc += __shfl_xor_sync(kFull, acc, 1);
    acc += __shfl_xor_sync(kFull, acc, 2);
    return (float)acc;
}

// Q4_1: value d * q + m (cpu.go:181-200): sum d * sum(q x) + m * sum(x).
__device__ __forceinline__ float dot_q4_1(const uint8_t *__restrict__ tile, int nb, const float *__restrict__ xs,
                                          int lane) {
    const int r = lane >> 2, q = lane & 3;
    const uint32_t *qw = reinterpret_cast<const uint32_t *>(tile) + r * 4 + q;
    const __half *dp = reinterpret_cast<const __half *>(tile + (size_t)nb * 128) + r;
    const __half *mp = dp + nb * 8;
    const float *xp = xs + 4 * q;
    constexpr float kOff = 8388608.f;  // 2^23
    double acc = 0.0;
#pragma unroll 2
    for (int b = 0; b < nb; ++b) {
        const uint32_t w = __ldg(qw + b * 32);
        const float d = __half2float(__ldg(dp + b * 8));
        const float mn = __half2float(__ldg(mp + b * 8));
        const float4 x0 = *reinterpret_cast<const float4 *>(xp + b * 32);
        const float4 x1 = *reinterpret_cast<const float4 *>(xp + b * 32 + 16);
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        float s = (b2f(lo, 0) - kOff) * x0.x;
        s = fmaf(b2f(hi, 0) - kOff, x1.x, s);
        s = fmaf(b2f(lo, 1) - kOff, x0.y, s);
        s = fmaf(b2f(hi, 1) - kOff, x1.y, s);
        s = fmaf(b2f(lo, 2) - kOff, x0.z, s);
        s = fmaf(b2f(hi, 2) - kOff, x1.z, s);
        s = fmaf(b2f(lo, 3) - kOff, x0.w, s);
        s = fmaf(b2f(hi, 3) - kOff, x1.w, s);
        const float sx = ((x0.x + x0.y) + (x0.z + x0.w)) + ((x1.x + x1.y) + (x1.z + x1.w));
        acc = fma((double)d, (double)s, fma((double)mn, (double)sx, acc));
    }
    acc += __shfl_xor_sync(kFull, acc, 1);
    acc += __shfl_xor_sync(kFull, acc, 2);
    return (float)acc;
}

// Q8_0: value d * int8 (cpu.go:201-215).  Lane q owns bytes 8q..8q+7.
__device__ __forceinline__ float dot_q8_0(const uint8_t *__restrict__ tile, int nb, const float *__restrict__ xs,
                                          int lane) {
    const int r = lane >> 2, q = lane & 3;
    const uint2 *qw = reinterpret_cast<const uint2 *>(tile) + r * 4 + q;
    const __half *dp = reinterpret_cast<const __half *>(tile + (size_t)nb * 256) + r;
    const float *xp = xs + 8 * q;
    constexpr float kOff = 8388736.f;  // 2^23 + 128: bytes are biased by 128
    double acc = 0.0;
#pragma unroll 2
    for (int b = 0; b < nb; ++b) {
        const uint2 w = __ldg(qw + b * 32);
        const float d = __half2float(__ldg(dp + b * 8));
        const float4 x0 = *reinterpret_cast<const float4 *>(xp + b * 32);
        const float4 x1 = *reinterpret_cast<const float4 *>(xp + b * 32 + 4);
        const uint32_t u0 = w.x ^ 0x80808080u, u1 = w.y ^ 0x80808080u;
        float s = (b2f(u0, 0) - kOff) * x0.x;
        s = fmaf(b2f(u0, 1) - kOff, x0.y, s);
        s = fmaf(b2f(u0, 2) - kOff, x0.z, s);
        s = fmaf(b2f(u0, 3) - kOff, x0.w, s);
        s = fmaf(b2f(u1, 0) - kOff, x1.x, s);
        s = fmaf(b2f(u1, 1) - kOff, x1.y, s);
        s = fmaf(b2f(u1, 2) - kOff, x1.z, s);
        s = fmaf(b2f(u1, 3) - kOff, x1.w, s);
        acc = fma((double)d, (double)s, acc);
    }
    acc += __shfl_xor_sync(kFull, acc, 1);
    acc += __shfl_xor_sync(kFull, acc, 2);
    return (float)acc;
}

__device__ __forceinline__ float tile_dot(const QMat &m, int tile, const float *xs, int lane) {
    const uint8_t *t = m.tiles + (size_t)tile * m.tile_bytes;
    switch (m.type) {
    case 3: return dot_q4_1(t, m.nb, xs, lane);
    case 8: return dot_q8_0(t, m.nb, xs, lane);
    default: return dot_q4_0(t, m.nb, xs, lane);
    }
}

// Element e of row `row` of a tile-layout matrix, dequantised (the embedding
// gather, kernels.go:19-73 / cpu.go:231-254).
__device__ __forceinline__ float gather(const QMat &m, int row, int e) {
    const uint8_t *t = m.tiles + (size_t)(row >> 3) * m.tile_bytes;
    const int r = row & 7, b = e >> 5, j = e & 31;
    const int qb = m.type == 8 ? 32 : 16;
    const float d = __half2float(reinterpret_cast<const __half *>(t + (size_t)m.nb * 8 * qb)[b * 8 + r]);
    const uint8_t *qs = t + ((size_t)b * 8 + r) * qb;
    if (m.type == 8) return d * (float)(int8_t)qs[j];
    const uint8_t byte = qs[j & 15];
    const int nib = j < 16 ? (byte & 15) : (byte >> 4);
    return d * (float)(nib - 8);
}

// RMSNorm of x (global, n floats) into hs (shared), cpu.go:81-98: the scale
// 1/sqrt(mean + eps) in double, then (x * s) * w.
__device__ __forceinline__ void rmsnorm_to_smem(const float *xs_in, const float *__restrict__ w, int n, float eps,
                                                float *hs, float *red) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += kThreads) {
        const float v = xs_in[i];
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float t = __fadd_rn(__fdiv_rn(ss, (float)n), eps);
    const float s = (float)(1.0 / sqrt((double)t));
    for (int i = threadIdx.x; i < n; i += kThreads) hs[i] = __fmul_rn(__fmul_rn(xs_in[i], s), __ldg(w + i));
    __syncthreads();
}

// ------------------------------------------------------------- phases --
// Work items are spread over CTAs first: tile i belongs to CTA i % ncta,
// warp (i / ncta) % kWarps, so a phase with few tiles still uses many SMs.

struct Smem {
    float *vec;  // max(embd, ff) floats
    float *red;  // reduction scratch
};

__device__ __forceinline__ bool cta_has_tiles(int cta, int ntiles) { return cta < ntiles; }

// Layer l's KV cache for token t: the model's own, or its slot of a batch's arena.
__device__ __forceinline__ float *kv_of(const DevModel &dm, const TokBatch *tb, int l, int t) {
    if (!tb) return dm.layer[l].kv;
    return tb->kv + ((size_t)tb->slot[t] * tb->layers + l) * 2 * (size_t)dm.ctx * dm.kvd;
}

// K1: RMSNorm + [Wq; Wk; Wv] + bias + RoPE + KV append for token t at
// position pos (kernels_fused.go:47-73,212-224; cpu.go:279-303).  With
// from_embed the residual is first taken from the embedding row of tok, and
// CTA 0 writes it to x.
__device__ void phase_qkv(const DevModel &dm, int l, int t, int pos, int tok, bool from_embed, float *kv, int cta,
                          int ncta, const Smem &sm) {
    const Layer &L = dm.layer[l];
    const int nq = L.q.rows >> 3, nk = L.k.rows >> 3, nv = L.v.rows >> 3, total = nq + nk + nv;
    if (!cta_has_tiles(cta, total)) return;
    const int E = dm.embd, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *xrow = dm.x + (size_t)t * E;
    float *xs = sm.vec + E;  // raw residual (second half of the buffer)
    if (from_embed) {
        for (int e = threadIdx.x; e < E; e += kThreads) {
            const float v = gather(dm.embed, tok, e);
            xs[e] = v;
            if (cta == 0) xrow[e] = v;
        }
    } else {
        for (int e = threadIdx.x; e < E; e += kThreads) xs[e] = __ldcg(xrow + e);
    }
    __syncthreads();
    rmsnorm_to_smem(xs, L.attn_norm, E, dm.eps, sm.vec, sm.red);
    const int hp = dm.head_dim >> 1;
    for (int tile = cta + ncta * warp; tile < total; tile += ncta * kWarps) {
        int seg, lt;
        const QMat *m;
        if (tile < nq) seg = 0, lt = tile, m = &L.q;
        else if (tile < nq + nk) seg = 1, lt = tile - nq, m = &L.k;
        else seg = 2, lt = tile - nq - nk, m = &L.v;
        float a = tile_dot(*m, lt, sm.vec, lane);
        const int r = lane >> 2, row = lt * 8 + r;
        const float *bias = seg == 0 ? L.bq : seg == 1 ? L.bk : L.bv;
        if (bias) a = __fadd_rn(a, __ldg(bias + row));
        if (seg < 2) {  // rotate adjacent pairs (rows 2p, 2p+1 of a head), cpu.go:371-385
            const float other = __shfl_xor_sync(kFull, a, 4);
            const int p = (row % dm.head_dim) >> 1;
            const float2 cs = __ldg(reinterpret_cast<const float2 *>(dm.rope_cs) + (size_t)pos * hp + p);
            if ((r & 1) == 0) a = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(other, cs.y));
            else a = __fadd_rn(__fmul_rn(other, cs.y), __fmul_rn(a, cs.x));
        }
        if ((lane & 3) == 0) {
            if (seg == 0) dm.q[(size_t)t * E + row] = a;
            else if (seg == 1) kv[(size_t)pos * dm.kvd + row] = a;
            else kv[((size_t)dm.ctx + pos) * dm.kvd + row] = a;
        }
    }
}

// K2 + the merge of K3: attention of token t (n positions visible) for item
// = (KV head g, chunk of kAttnChunk positions), for every query head of g's
// GQA group (cpu.go:304-335): the chunk's K and V rows are read once into
// shared memory and warp j computes query head j of the group, with no
// barrier between its steps: lane p scores positions p and p + 32 (f32 dot
// products, as cpu.go:311-316), the chunk max and exp-sum come from warp
// shuffles (exp in double, rounded to f32, as cpu.go:321), then lane d sums
// dimensions 2d, 2d + 1 of the exp-weighted V rows (kernels_fused.go:82-146).
// The last CTA of (token, group) to finish merges the chunks of the group's
// heads (kernels_fused.go:150-170) into att.  Groups of up to 8 query heads
// per KV head; more take several rounds of the warps.  With kDirect, a token
// whose n positions fit one chunk writes o / l into att itself, with no
// partials and no merge.
template <bool kDirect>
__device__ void phase_attn(const DevModel &dm, const float *kv, int t, int n, int hist_end, int item, uint32_t *att_cnt,
                           const Smem &sm) {
    const int HD = dm.head_dim, grp = dm.heads / dm.kv_heads;
    const int nch = (n + kAttnChunk - 1) / kAttnChunk;
    const int g = item / nch, c = item % nch;
    const int KS = HD + 4;                       // shared row stride
    float *ks = sm.vec;                          // [kAttnChunk][KS]
    float *vs = ks + kAttnChunk * KS;            // [kAttnChunk][KS]
    float *qg = vs + kAttnChunk * KS;            // [grp][HD]
    __shared__ int last;
    const int p0 = c * kAttnChunk, cnt = min(kAttnChunk, n - p0);
    const int nd4 = HD / 4;
    // the chunk's K and V rows and the group's queries by asynchronous 16-byte copies, all in flight at once.
    // Rows below hist_end were written by earlier launches, so their copies start before the wait for the
    // QKV product (a programmatic dependency: it writes this launch's rows and the queries); the rest after.
    const int pe = min(cnt, max(0, hist_end - p0));
    auto copy_rows = [&](int i0, int i1) {
        for (int i = i0 + (int)threadIdx.x; i < i1; i += kThreads) {
            const int p = i / nd4, d4 = i % nd4;
            const size_t row = (size_t)(p0 + p) * dm.kvd + g * HD;
            cp_async16(ks + p * KS + d4 * 4, kv + row + 4 * d4);
            cp_async16(vs + p * KS + d4 * 4, kv + (size_t)dm.ctx * dm.kvd + row + 4 * d4);
        }
    };
    copy_rows(0, pe * nd4);
    // wait for the QKV product, then let the output product start its set-up as this grid's last CTAs run
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    copy_rows(pe * nd4, cnt * nd4);
    for (int i = threadIdx.x; i < grp * nd4; i += kThreads)
        cp_async16(qg + 4 * i, dm.q + (size_t)t * dm.embd + g * grp * HD + 4 * i);
    asm volatile("cp.async.commit_group;\n cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < grp; j += kWarps) {
        const int h = g * grp + j;
        const float *qh = qg + j * HD;
        float s[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int p = lane + 32 * k;
            float a0 = 0.f, a1 = 0.f;
            if (p < cnt) {
                const float *kr = ks + p * KS;
                for (int d = 0; d < HD; d += 4) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(kr + d);
                    const float4 q4 = *reinterpret_cast<const float4 *>(qh + d);
                    a0 = fmaf(q4.x, k4.x, a0);
                    a1 = fmaf(q4.y, k4.y, a1);
                    a0 = fmaf(q4.z, k4.z, a0);
                    a1 = fmaf(q4.w, k4.w, a1);
                }
            }
            s[k] = p < cnt ? __fmul_rn(a0 + a1, dm.scale) : -FLT_MAX;
        }
        const float mx = warp_max(fmaxf(s[0], s[1]));
        float e[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) e[k] = lane + 32 * k < cnt ? (float)exp((double)__fsub_rn(s[k], mx)) : 0.f;
        const float lsum = warp_sum(e[0] + e[1]);
        // V: lane covers dimensions 2 lane, 2 lane + 1 (and 64 + 2 lane, 65 + 2 lane for head_dim 128)
        const bool two = HD > 64;
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
        for (int p = 0; p < cnt; ++p) {
            const float w = __shfl_sync(kFull, p < 32 ? e[0] : e[1], p & 31);
            const float2 va = *reinterpret_cast<const float2 *>(vs + p * KS + 2 * lane);
            o0 = fmaf(w, va.x, o0);
            o1 = fmaf(w, va.y, o1);
            if (two) {
                const float2 vb = *reinterpret_cast<const float2 *>(vs + p * KS + 64 + 2 * lane);
                o2 = fmaf(w, vb.x, o2);
                o3 = fmaf(w, vb.y, o3);
            }
        }
        const size_t th = (size_t)t * dm.heads + h;
        if constexpr (kDirect) {
            // the whole context in one chunk: o / l straight into att (by the reciprocal: within 1.5 ulp of
            // the merge's correctly rounded quotient), with no partials and no merge; else the partials
            const bool direct = nch == 1;
            const float r = direct ? __frcp_rn(lsum) : 1.f;
            float *dst = direct ? dm.att + (size_t)t * dm.embd + h * HD + 2 * lane
                                : dm.part_pv + (th * dm.nchunk + c) * HD + 2 * lane;
            dst[0] = __fmul_rn(o0, r), dst[1] = __fmul_rn(o1, r);
            if (two) dst[64] = __fmul_rn(o2, r), dst[65] = __fmul_rn(o3, r);
            if (!direct && lane == 0) dm.part_ml[th * dm.nchunk + c] = make_float2(mx, lsum);
        } else {
            float *pv = dm.part_pv + (th * dm.nchunk + c) * HD + 2 * lane;
            pv[0] = o0, pv[1] = o1;
            if (two) pv[64] = o2, pv[65] = o3;
            if (lane == 0) dm.part_ml[th * dm.nchunk + c] = make_float2(mx, lsum);
        }
    }
    if (kDirect && nch == 1) return;  // no partials, no merge
    // the last arriving CTA of this (token, group) merges the group's heads
    __syncthreads();
    const size_t tg = (size_t)t * dm.kv_heads + g;
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(att_cnt + tg, 1u);
        last = prev == (unsigned)(nch - 1);
        if (last) att_cnt[tg] = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // per head j: the chunks' weights f[j][c] = exp(max_c - M) (double) and the sum of f * l (over the lanes,
    // then a fixed shuffle tree), computed once in the K/V rows' shared memory (free now); then each (head,
    // dimension) folds the chunks' partial sums in chunk order with 8 chunks' loads in flight.  (Up to 2
    // chunks, or a context whose weights do not fit, each thread computes the weights itself.)
    double *fw = reinterpret_cast<double *>(sm.vec), *lt = fw + (size_t)grp * nch;
    const bool fit = nch > 2 && (size_t)grp * (nch + 1) * sizeof(double) <= (size_t)2 * kAttnChunk * KS * sizeof(float);
    // one (head, dimension) per thread: its first kPre chunks' partial sums are requested before the weights
    // are computed, so that the two rounds of loads overlap
    constexpr int kPre = 4;
    const bool one = fit && grp * HD <= kThreads;
    float pre[kPre];
    if (one && (int)threadIdx.x < grp * HD) {
        const int j = threadIdx.x / HD, d = threadIdx.x % HD;
        const float *pv = dm.part_pv + ((size_t)t * dm.heads + g * grp + j) * dm.nchunk * HD + d;
#pragma unroll
        for (int k = 0; k < kPre; ++k) pre[k] = k < nch ? __ldcg(pv + (size_t)k * HD) : 0.f;
    }
    if (fit) {
        for (int j = warp; j < grp; j += kWarps) {
            const size_t th = (size_t)t * dm.heads + g * grp + j;
            float M = -FLT_MAX;
            float2 ml0 = make_float2(-FLT_MAX, 0.f);  // this lane's first chunk (most contexts have at most 32)
            if (lane < nch) ml0 = __ldcg(&dm.part_ml[th * dm.nchunk + lane]);
            M = ml0.x;
            for (int cc = lane + 32; cc < nch; cc += 32) M = fmaxf(M, __ldcg(&dm.part_ml[th * dm.nchunk + cc].x));
            M = warp_max(M);
            // the weights and the sum of f * l over the chunks (lanes, then a fixed shuffle tree)
            double l = 0.0;
            for (int cc = lane; cc < nch; cc += 32) {
                const float2 ml = cc == lane ? ml0 : __ldcg(&dm.part_ml[th * dm.nchunk + cc]);
                const double f = exp((double)ml.x - (double)M);
                fw[j * nch + cc] = f;
                l = fma(f, (double)ml.y, l);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(kFull, l, o);
            if (lane == 0) lt[j] = l;
        }
        __syncthreads();
    }
    if (one) {
        if ((int)threadIdx.x < grp * HD) {
            const int j = threadIdx.x / HD, d = threadIdx.x % HD, h = g * grp + j;
            const float *pv = dm.part_pv + ((size_t)t * dm.heads + h) * dm.nchunk * HD + d;
            double ot = 0.0;
#pragma unroll
            for (int k = 0; k < kPre; ++k)
                if (k < nch) ot = fma(fw[j * nch + k], (double)pre[k], ot);
            for (int c0 = kPre; c0 < nch; c0 += 8) {  // the rest, 8 chunks' loads in flight
                float v8[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v8[k] = c0 + k < nch ? __ldcg(pv + (size_t)(c0 + k) * HD) : 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (c0 + k < nch) ot = fma(fw[j * nch + c0 + k], (double)v8[k], ot);
            }
            dm.att[(size_t)t * dm.embd + h * HD + d] = (float)(ot / lt[j]);
        }
        return;
    }
    for (int i = threadIdx.x; i < grp * HD; i += kThreads) {
        const int j = i / HD, d = i % HD, h = g * grp + j;
        const size_t th = (size_t)t * dm.heads + h;
        const float *pv = dm.part_pv + th * dm.nchunk * HD + d;
        double ot = 0.0, l = 0.0;
        if (fit) {
            for (int c0 = 0; c0 < nch; c0 += 8) {
                float v8[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v8[k] = c0 + k < nch ? __ldcg(pv + (size_t)(c0 + k) * HD) : 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (c0 + k < nch) ot = fma(fw[j * nch + c0 + k], (double)v8[k], ot);
            }
            l = lt[j];
        } else {
            float M = -FLT_MAX;
            for (int cc = 0; cc < nch; ++cc) M = fmaxf(M, __ldcg(&dm.part_ml[th * dm.nchunk + cc].x));
            for (int cc = 0; cc < nch; ++cc) {
                const float2 ml = __ldcg(&dm.part_ml[th * dm.nchunk + cc]);
                const double f = exp((double)ml.x - (double)M);
                l = fma(f, (double)ml.y, l);
                ot = fma(f, (double)__ldcg(pv + (size_t)cc * HD), ot);
            }
        }
        dm.att[(size_t)t * dm.embd + h * HD + d] = (float)(ot / l);
    }
}

// K3's product: x += Wo att (cpu.go:336-339).
__device__ void phase_oproj(const DevModel &dm, int l, int t, int cta, int ncta, const Smem &sm) {
    const Layer &L = dm.layer[l];
    const int ntiles = L.o.rows >> 3;
    if (!cta_has_tiles(cta, ntiles)) return;
    const int E = dm.embd, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < E; i += kThreads) sm.vec[i] = __ldcg(dm.att + (size_t)t * E + i);
    __syncthreads();
    float *xrow = dm.x + (size_t)t * E;
    for (int tile = cta + ncta * warp; tile < ntiles; tile += ncta * kWarps) {
        const float a = tile_dot(L.o, tile, sm.vec, lane);
        const int row = tile * 8 + (lane >> 2);
        if ((lane & 3) == 0) xrow[row] = __fadd_rn(__ldcg(xrow + row), a);
    }
}

// K4: RMSNorm + [Wgate; Wup] + SwiGLU (kernels_fused.go:28-42; cpu.go
// :340-346): act = g / (1 + exp(-g)) * u, exp in double.
__device__ void phase_gateup(const DevModel &dm, int l, int t, int cta, int ncta, const Smem &sm) {
    const Layer &L = dm.layer[l];
    const int ntiles = L.gate.rows >> 3;
    if (!cta_has_tiles(cta, ntiles)) return;
    const int E = dm.embd, F = dm.ff, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *xs = sm.vec + E;
    for (int e = threadIdx.x; e < E; e += kThreads) xs[e] = __ldcg(dm.x + (size_t)t * E + e);
    __syncthreads();
    rmsnorm_to_smem(xs, L.ffn_norm, E, dm.eps, sm.vec, sm.red);
    for (int tile = cta + ncta * warp; tile < ntiles; tile += ncta * kWarps) {
        const float g = tile_dot(L.gate, tile, sm.vec, lane);
        const float u = tile_dot(L.up, tile, sm.vec, lane);
        const int row = tile * 8 + (lane >> 2);
        if ((lane & 3) == 0 && row < F) {
            const float den = __fadd_rn(1.f, (float)exp(-(double)g));
            dm.act[(size_t)t * F + row] = __fmul_rn(__fdiv_rn(g, den), u);
        }
    }
}

// K5: x += Wdown act (cpu.go:347-350).
__device__ void phase_down(const DevModel &dm, int l, int t, int cta, int ncta, const Smem &sm) {
    const Layer &L = dm.layer[l];
    const int ntiles = L.down.rows >> 3;
    if (!cta_has_tiles(cta, ntiles)) return;
    const int E = dm.embd, F = dm.ff, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < F; i += kThreads) sm.vec[i] = __ldcg(dm.act + (size_t)t * F + i);
    __syncthreads();
    float *xrow = dm.x + (size_t)t * E;
    for (int tile = cta + ncta * warp; tile < ntiles; tile += ncta * kWarps) {
        const float a = tile_dot(L.down, tile, sm.vec, lane);
        const int row = tile * 8 + (lane >> 2);
        if ((lane & 3) == 0) xrow[row] = __fadd_rn(__ldcg(xrow + row), a);
    }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// The head: RMSNorm(output_norm) of token t's residual, logits = Wout h
// (cpu.go:357-363), and this CTA's argmax partial (value, index).
__device__ void phase_head(const DevModel &dm, int t, int cta, int ncta, float *logits, float2 *am_part,
                           const Smem &sm) {
    const int E = dm.embd, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ntiles = dm.head.rows >> 3;
    float *xs = sm.vec + E;
    for (int e = threadIdx.x; e < E; e += kThreads) xs[e] = __ldcg(dm.x + (size_t)t * E + e);
    __syncthreads();
    rmsnorm_to_smem(xs, dm.out_norm, E, dm.eps, sm.vec, sm.red);
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int tile = cta + ncta * warp; tile < ntiles; tile += ncta * kWarps) {
        const float a = tile_dot(dm.head, tile, sm.vec, lane);
        const int row = tile * 8 + (lane >> 2);
        if (row < dm.vocab) {
            if (logits && (lane & 3) == 0) logits[row] = a;
            if (better(a, row, bv, bi)) bv = a, bi = row;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    __shared__ float wv[kWarps];
    __shared__ int wi[kWarps];
    if (lane == 0) wv[warp] = bv, wi[warp] = bi;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kWarps; ++w)
            if (better(wv[w], wi[w], bv, bi)) bv = wv[w], bi = wi[w];
        am_part[cta] = make_float2(bv, __int_as_float(bi));
    }
}

// The argmax over the CTAs' partials (first index of the largest value).
__device__ __forceinline__ int reduce_argmax(const float2 *am_part, int nparts) {
    __shared__ int result;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < nparts; i += kThreads) {
        const float2 p = __ldcg(am_part + i);
        const int pi = __float_as_int(p.y);
        if (better(p.x, pi, bv, bi)) bv = p.x, bi = pi;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    __shared__ float wv[kWarps];
    __shared__ int wi[kWarps];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) wv[warp] = bv, wi[warp] = bi;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kWarps; ++w)
            if (better(wv[w], wi[w], bv, bi)) bv = wv[w], bi = wi[w];
        result = bi == 0x7fffffff ? 0 : bi;
    }
    __syncthreads();
    return result;
}

__device__ __forceinline__ Smem smem_views(float *base, const DevModel &dm) { return Smem{base, base + dm.smem_vec}; }

// ---------------------------------------------------- per-phase kernels --

// The embedding rows of m tokens into x, and each row's sum of squares into
// ssq[t][0] (the tensor-core products' RMSNorm input; the other tiles' 0).
__global__ void __launch_bounds__(kThreads) k_embed(const DevModel *__restrict__ dmp, const TokBatch *tb) {
    const DevModel &dm = *dmp;
    const int t = blockIdx.x;
    const int tok = tb ? tb->tok[t] : dm.tokens[dm.state[1] + t];
    float ss = 0.f;
    for (int e = threadIdx.x; e < dm.embd; e += kThreads) {
        const float v = gather(dm.embed, tok, e);
        dm.x[(size_t)t * dm.embd + e] = v;
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    __shared__ float red[kWarps];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < kSsqTiles) {
        float v = 0.f;
        if (threadIdx.x == 0)
            for (int w = 0; w < kWarps; ++w) v += red[w];
        dm.ssq[(size_t)t * kSsqTiles + threadIdx.x] = v;
    }
}

__global__ void __launch_bounds__(kThreads) k_qkv(const DevModel *__restrict__ dmp, int l, const TokBatch *tb) {
    extern __shared__ float smem[];
    const DevModel &dm = *dmp;
    const int t = blockIdx.y;
    const int pos = tb ? tb->pos[t] : dm.state[0] + t;
    const int tok = l == 0 ? (tb ? tb->tok[t] : dm.tokens[dm.state[1] + t]) : 0;
    phase_qkv(dm, l, t, pos, tok, l == 0, kv_of(dm, tb, l, t), blockIdx.x, gridDim.x, smem_views(smem, dm));
}

// kDirect: a token whose context fits one chunk writes its output without partials or a merge (single-sequence
// chunks; measured slower for the multi-stream batches, which take k_attn<false>).
template <bool kDirect>
__global__ void __launch_bounds__(kThreads) k_attn(const DevModel *__restrict__ dmp, int l, const TokBatch *tb) {
    extern __shared__ float smem[];
    // Launched as a programmatic dependent of the QKV product, which writes the queries and this launch's K/V
    // rows; phase_attn waits for it (a no-op otherwise) after requesting the rows written before it.  The
    // positions and KV slots were written before the launch.
    const DevModel &dm = *dmp;
    const int t = blockIdx.y;
    const int n = (tb ? tb->pos[t] : dm.state[0] + t) + 1;
    const int nch = (n + kAttnChunk - 1) / kAttnChunk;
    if ((int)blockIdx.x >= dm.kv_heads * nch) return;
    // hist_end: the first position of token t's sequence that this launch writes (its lowest position among
    // the batch's tokens of the same KV slot; for one sequence, the chunk's first position)
    __shared__ int hist_end;
    if (threadIdx.x < 32) {
        int h = tb ? n - 1 : dm.state[0];
        if (tb) {
            const int slot = tb->slot[t];
            for (int u = threadIdx.x; u < (int)gridDim.y; u += 32)
                if (tb->slot[u] == slot) h = min(h, tb->pos[u]);
            for (int o = 16; o; o >>= 1) h = min(h, __shfl_xor_sync(kFull, h, o));
        }
        if (threadIdx.x == 0) hist_end = h;
    }
    __syncthreads();
    phase_attn<kDirect>(dm, kv_of(dm, tb, l, t), t, n, hist_end, blockIdx.x, dm.att_cnt, smem_views(smem, dm));
}

__global__ void __launch_bounds__(kThreads) k_oproj(const DevModel *__restrict__ dmp, int l) {
    extern __shared__ float smem[];
    phase_oproj(*dmp, l, blockIdx.y, blockIdx.x, gridDim.x, smem_views(smem, *dmp));
}

__global__ void __launch_bounds__(kThreads) k_gateup(const DevModel *__restrict__ dmp, int l) {
    extern __shared__ float smem[];
    phase_gateup(*dmp, l, blockIdx.y, blockIdx.x, gridDim.x, smem_views(smem, *dmp));
}

__global__ void __launch_bounds__(kThreads) k_down(const DevModel *__restrict__ dmp, int l) {
    extern __shared__ float smem[];
    phase_down(*dmp, l, blockIdx.y, blockIdx.x, gridDim.x, smem_views(smem, *dmp));
}

// The head and the argmax: the last CTA to finish reduces the partials,
// writes the token and advances the state (kernels.go:354-415).
__global__ void __launch_bounds__(kThreads) k_head(const DevModel *__restrict__ dmp, int t_src, int adv) {
    extern __shared__ float smem[];
    const DevModel &dm = *dmp;
    Smem sm = smem_views(smem, dm);
    phase_head(dm, t_src, blockIdx.x, gridDim.x, dm.logits, dm.am_part, sm);
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(dm.am_count, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int tok = reduce_argmax(dm.am_part, gridDim.x);
    if (threadIdx.x == 0) {
        *dm.am_count = 0;
        const uint32_t step = dm.state[1] + adv;
        dm.tokens[step] = tok;
        dm.state[0] += adv;
        dm.state[1] = step;
    }
}

// The batch head: for row j = blockIdx.y, the argmax of token head_rows[j]
// into out[j] (per-row partials and arrival counters; no logits are kept).
__global__ void __launch_bounds__(kThreads) k_head_batch(const DevModel *__restrict__ dmp, TokBatch *tb) {
    extern __shared__ float smem[];
    const DevModel &dm = *dmp;
    Smem sm = smem_views(smem, dm);
    const int j = blockIdx.y;
    float2 *part = dm.am_part + (size_t)j * gridDim.x;
    phase_head(dm, tb->head_rows[j], blockIdx.x, gridDim.x, nullptr, part, sm);
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(dm.am_count + j, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int tok = reduce_argmax(part, gridDim.x);
    if (threadIdx.x == 0) {
        dm.am_count[j] = 0;
        tb->out[j] = tok;
    }
}

__global__ void k_advance(const DevModel *__restrict__ dmp, int n) {
    dmp->state[0] += n;
    dmp->state[1] += n;
}

// ------------------------------------------------------------ loading --

__device__ __forceinline__ int neox_map(int nr, int hd) {  // fused.go:331-334
    const int h = nr / hd, k = nr % hd;
    return h * hd + k / 2 + (k % 2) * (hd / 2);
}

__global__ void k_repack(const uint8_t *__restrict__ raw, int rows, int nb, int type, uint8_t *__restrict__ tiles,
                         int tile_bytes, int dst_row0, int neox_hd) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)rows * nb) return;
    const int rr = (int)(idx / nb), b = (int)(idx % nb);
    const int src = neox_hd > 0 ? neox_map(rr, neox_hd) : rr;
    const int bb = type == 8 ? 34 : type == 3 ? 20 : 18;
    const int qb = type == 8 ? 32 : 16, qoff = type == 3 ? 4 : 2;
    const uint8_t *blk = raw + ((size_t)src * nb + b) * bb;
    const int drow = dst_row0 + rr, r = drow & 7;
    uint8_t *tp = tiles + (size_t)(drow >> 3) * tile_bytes;
    uint8_t *qd = tp + ((size_t)b * 8 + r) * qb;
    for (int j = 0; j < qb; ++j) qd[j] = blk[qoff + j];
    uint8_t *dd = tp + (size_t)nb * 8 * qb + ((size_t)b * 8 + r) * 2;
    dd[0] = blk[0], dd[1] = blk[1];
    if (type == 3) {
        uint8_t *md = tp + (size_t)nb * 8 * qb + (size_t)nb * 16 + ((size_t)b * 8 + r) * 2;
        md[0] = blk[2], md[1] = blk[3];
    }
}

}  // namespace

// ---------------------------------------------------------- launchers --

int smem_vec_floats(const Shapes &s) {
    const int vec = s.embd + (s.embd > s.ff ? s.embd : s.ff);
    // attention: K and V chunks, the group's queries
    const int attn = 2 * kAttnChunk * (s.head_dim + 4) + (s.heads / s.kv_heads) * s.head_dim;
    return vec > attn ? vec : attn;
}

size_t smem_bytes(const Shapes &s) { return ((size_t)smem_vec_floats(s) + 2 * kWarps) * sizeof(float); }

cudaError_t prepare_kernels(const Shapes &s) {
    // the attribute is per function, for the whole process: only ever raise it, so that
    // opening a smaller model does not break the kernels of a larger one still open
    static std::mutex mu;
    static int set = 0;
    std::lock_guard<std::mutex> lock(mu);
    const int sh = std::max(set, (int)smem_bytes(s));
    if (sh == set) return cudaSuccess;
    set = sh;
    cudaError_t e = cudaSuccess;
    for (const void *k : {(const void *)k_qkv, (const void *)k_attn<true>, (const void *)k_attn<false>,
                          (const void *)k_oproj, (const void *)k_gateup, (const void *)k_down, (const void *)k_head,
                          (const void *)k_head_batch})
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, sh);
    return e;
}

void launch_repack(const uint8_t *raw, int rows, int nb, int type, uint8_t *tiles, int tile_bytes, int dst_row0,
                   int neox_hd, cudaStream_t st) {
    const int64_t n = (int64_t)rows * nb;
    k_repack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(raw, rows, nb, type, tiles, tile_bytes, dst_row0, neox_hd);
}

void launch_embed(const DevModel *dm, const Shapes &s, int m, cudaStream_t st, const TokBatch *tb) {
    k_embed<<<m, kThreads, 0, st>>>(dm, tb);
}

static inline unsigned ctas_for(int tiles) { return (unsigned)((tiles + kWarps - 1) / kWarps); }

void launch_layer(const DevModel *dm, const Shapes &s, int l, int m, cudaStream_t st, const TokBatch *tb) {
    const size_t sh = smem_bytes(s);
    k_qkv<<<dim3(ctas_for(s.qkv_tiles), m), kThreads, sh, st>>>(dm, l, tb);
    if (tb) k_attn<false><<<dim3(s.kv_heads * s.nchunk, m), kThreads, sh, st>>>(dm, l, tb);
    else k_attn<true><<<dim3(s.kv_heads * s.nchunk, m), kThreads, sh, st>>>(dm, l, tb);
    k_oproj<<<dim3(ctas_for(s.o_tiles), m), kThreads, sh, st>>>(dm, l);
    k_gateup<<<dim3(ctas_for(s.gu_tiles), m), kThreads, sh, st>>>(dm, l);
    k_down<<<dim3(ctas_for(s.down_tiles), m), kThreads, sh, st>>>(dm, l);
}

void launch_head(const DevModel *dm, const Shapes &s, int t_src, int adv, cudaStream_t st) {
    k_head<<<s.head_ctas, kThreads, smem_bytes(s), st>>>(dm, t_src, adv);
}

cudaError_t launch_attention(const DevModel *dm, const Shapes &s, int l, int m, cudaStream_t st, const TokBatch *tb,
                             bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(s.kv_heads * s.nchunk, m);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes(s);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return tb ? cudaLaunchKernelEx(&cfg, k_attn<false>, dm, l, tb) : cudaLaunchKernelEx(&cfg, k_attn<true>, dm, l, tb);
}

void launch_head_batch(const DevModel *dm, const Shapes &s, TokBatch *tb, int rows, cudaStream_t st) {
    k_head_batch<<<dim3(s.head_ctas, rows), kThreads, smem_bytes(s), st>>>(dm, tb);
}

void launch_advance(const DevModel *dm, int n, cudaStream_t st) { k_advance<<<1, 1, 0, st>>>(dm, n); }

}  // namespace llmb
