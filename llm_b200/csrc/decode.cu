// The persistent decode kernel: DecodeBatch tokens of batch-1 greedy decoding
// in one cooperative launch over every SM (Generate's decode submits,
// gpu.go:987-1009, and the per-token pass, gpu.go:792-832, fused.go:259-289).
//
// Structure of a CTA (one per SM, 8 warps, so up to 255 registers a thread):
//   - the CTA's weight tiles stream, in the order the CTA consumes them,
//     through a ring of shared-memory slots with 1D bulk TMA copies into
//     this CTA's own shared memory, tracked by mbarriers.  One thread issues
//     them and refills each slot as soon as its unit is consumed.  Weights do
//     not depend on activations, so the stream runs ahead across phases,
//     layers and tokens as far as the ring allows;
//   - the 8 warps compute (paired f32 math): a row per warp for units of one
//     tile, a tile's blocks split across warps for larger units; partials
//     meet in shared memory and shuffles in a fixed order, so results are
//     deterministic.
//
// Activations move between CTAs as 64-bit words {f32 value, u32 tag}
// written and polled with relaxed GPU-scope accesses (a value and its tag
// are one single-copy-atomic store, so a reader that sees the tag sees the
// value): each CTA waits only for the vector it needs, with no grid-wide
// barrier between phases.  A tag is unique per (token, layer, phase)
// across calls (a device epoch counter).  A token ends with each CTA's argmax
// partial published the same way after a release fence, and read by every
// CTA, then an acquire fence: that also makes the token's KV-cache rows
// visible to the next token's attention, with no grid-wide barrier.
//
// Every wait (mbarrier, tag poll) is bounded: past its limit
// the kernel records an error in DevModel::err and returns; the CTA first
// waits (bounded) for its weight copies in flight.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>

#include "kernels.hpp"

namespace llmb {

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kCons = 8;                 // consumer warps
constexpr int kConsThreads = kCons * 32; // 256
constexpr int kDecThreads = kConsThreads;  // 8 warps: 2 per SM sub-partition, up to 255 registers each
constexpr int kFeeder = kConsThreads - 1;  // the thread that issues the weight ring's copies
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: the default limit of every wait
#ifndef LLMB_POLL_SLEEP_NS
#define LLMB_POLL_SLEEP_NS 0
#endif
constexpr unsigned kPollSleepNs = LLMB_POLL_SLEEP_NS;

// ------------------------------------------------------------ primitives --

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-space loads at 32-bit shared addresses: the dot products' operands
// sit in shared memory but reach them through generic pointers kept in
// structs, which the compiler cannot prove shared (generic loads measured
// 10-25 % slower in these products).
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds_u64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float lds_h2f(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return __half2float(__ushort_as_half(v));
}
__device__ __forceinline__ float4 lds_f4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}

// 1D bulk copy global -> this CTA's shared memory, completing on mbarrier b.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *b) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(b))
                 : "memory");
}

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsThreads) : "memory"); }

// A consumer barrier that also ORs a predicate over the consumer threads, so
// that every thread takes the same branch after it (a thread that left a
// named barrier early would leave the others waiting).
__device__ __forceinline__ bool cons_or(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(kConsThreads)
        : "memory");
    return r != 0;
}

// Two consecutive tagged words (each single-copy atomic on its own).
__device__ __forceinline__ void ld_relaxed2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// L2 loads as volatile asm: issued where written (before a wait), not sunk to their first use.
__device__ __forceinline__ float4 ld_cg_early(const float4 *p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ float2 ld_cg_early(const float2 *p) {
    float2 v;
    asm volatile("ld.global.cg.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
    return v;
}

__device__ __forceinline__ void st_relaxed(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void ll_put(uint64_t *p, float v, uint32_t tag) {
    st_relaxed(p, (uint64_t)tag << 32 | __float_as_uint(v));
}

__device__ __forceinline__ int read_err(const int *e) { return *(volatile const int *)e; }

// The limit of every wait of this launch, in ns (DecParams::wait_ns, or
// kWaitNs), set once by thread 0 before the first barrier.
__shared__ uint64_t s_wait_ns;

// A tagged vector to poll into shared memory: src[0, n) (n even), tag, dst.
struct Seg {
    const uint64_t *src;
    int n;
    uint32_t tag;
    float *dst;
};

// Polls up to 3 tagged vectors.  Each consumer thread owns word pairs t,
// t + 256, ... of their concatenation.  It polls them in rounds of up to 4
// pairs: every round issues the loads of all pairs still pending before
// testing any, so once the data is written a thread sees all of it within
// about one L2 round trip (a pair-by-pair wait would pay one round trip per
// pair that was stale when loaded).  Without a back-off sleep a 576-float
// vector written by 72 CTAs reaches all 148 CTAs in about 1.0 us on B200,
// against 1.6 us with a 64 ns sleep.
__device__ __forceinline__ const uint64_t *seg_src(const Seg *sg, int ns, int i, int &j, int &lo) {
    lo = 0;
    for (j = 0; j < ns; ++j) {
        const int np = sg[j].n >> 1;
        if (i < lo + np) return sg[j].src + 2 * (i - lo);
        lo += np;
    }
    return nullptr;
}

template <int NS>
__device__ __noinline__ bool poll_segs(const Seg (&sg)[NS], int *err) {
    int npairs = 0;
#pragma unroll
    for (int j = 0; j < NS; ++j) npairs += sg[j].n >> 1;
    constexpr int K = 4;
    for (int base = 0; base < npairs; base += K * kConsThreads) {
        uint64_t v[2 * K];
        unsigned pend = 0;
#pragma unroll
        for (int k = 0; k < K; ++k)
            if (base + threadIdx.x + k * kConsThreads < npairs) pend |= 1u << k;
        const uint64_t t0 = gtimer();
        unsigned spins = 0;
        while (pend) {
#pragma unroll
            for (int k = 0; k < K; ++k) {
                if (!(pend >> k & 1)) continue;
                int j, lo;
                ld_relaxed2(seg_src(sg, NS, base + threadIdx.x + k * kConsThreads, j, lo), v[2 * k], v[2 * k + 1]);
            }
#pragma unroll
            for (int k = 0; k < K; ++k) {
                if (!(pend >> k & 1)) continue;
                const int i = base + threadIdx.x + k * kConsThreads;
                int j, lo;
                seg_src(sg, NS, i, j, lo);
                const uint32_t tag = sg[j].tag;
                if ((uint32_t)(v[2 * k] >> 32) == tag && (uint32_t)(v[2 * k + 1] >> 32) == tag) {
                    float *d = sg[j].dst + 2 * (i - lo);
                    d[0] = __uint_as_float((uint32_t)v[2 * k]);
                    d[1] = __uint_as_float((uint32_t)v[2 * k + 1]);
                    pend &= ~(1u << k);
                }
            }
            if (pend) {
                if (kPollSleepNs) __nanosleep(kPollSleepNs);
                if ((++spins & 255) == 0) {
                    if (read_err(err)) return false;
                    if (gtimer() - t0 > s_wait_ns) {
                        atomicExch(err, DEV_TAG_TIMEOUT);
                        return false;
                    }
                }
            }
        }
    }
    return true;
}

__device__ __forceinline__ bool poll_two(const uint64_t *a, int na, uint32_t ta, float *da, const uint64_t *b, int nb,
                                         uint32_t tb, float *db, int *err) {
    const Seg sg[2] = {{a, na, ta, da}, {b, nb, tb, db}};
    return poll_segs(sg, err);
}

__device__ __forceinline__ float b2f(uint32_t v, int k) {
    return __int_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | k));
}

// Phase timeline (DevModel::trace): for event ev of this CTA, stamps 0..2
// (entry, input ready, exit, globaltimer ns) and the SM cycles the phase
// spent waiting for weight slots (field 3, accumulated by unit_rows).
__shared__ uint64_t s_ring_wait;

struct Trace {
    uint64_t *p;  // this CTA's events, or null
    __device__ void stamp(int ev, int k) const {
        if (p && threadIdx.x == 0) {
            p[ev * 4 + k] = gtimer();
            if (k == 2) p[ev * 4 + 3] = s_ring_wait, s_ring_wait = 0;
        }
    }
};

// ------------------------------------------------------------ schedule --
// The CTA's share of a matrix: tiles [a, b) (contiguous), in units of at most
// `per` tiles (one bulk copy each, at most one slot).

struct Share {
    int a, b, per;
};

// floor(T * i / P) for the split of T tiles over P CTAs: 32-bit unsigned
// arithmetic (T * P stays far below 2^32), since a 64-bit division is a
// long dependent sequence that sat at the head of every phase.
__device__ __forceinline__ int split_at(int T, int i, int P) { return (int)((unsigned)T * (unsigned)i / (unsigned)P); }

// The CTA's share of each kind of matrix, computed once per launch: the rows
// of a kind are the same in every layer, and `per` depends only on the
// format.  (Integer divisions are long dependent sequences; at the head of a
// phase they delayed its first poll.)
enum { SK_QKV = 0, SK_O, SK_GU, SK_DOWN, SK_HEAD, SK_N };
struct ShareTab {
    int a[SK_N], b[SK_N];  // tiles [a, b) of the kind (QKV: of q, k, v in turn; down: half tiles if down_half)
    int per[SK_N][3];      // tiles per unit by format: Q4_0, Q4_1, Q8_0
    int down_half;         // the down product in half tiles (4 rows) per CTA
};
static_assert(sizeof(ShareTab) <= 128, "the shared-memory layout reserves 128 bytes");

__device__ __forceinline__ int fmt_ix(int type) { return type == 8 ? 2 : type == 3 ? 1 : 0; }

// The down product runs in half tiles (4 rows, two warps per row) when the
// grid has a CTA for each: its rows are the longest (ff weights), and half the
// CTAs had no down rows.
__device__ __forceinline__ bool down_halves(const QMat &down, int ncta) { return 2 * (down.rows >> 3) <= ncta; }

__device__ __forceinline__ Share share(const QMat &m, int cta, int ncta, int slot_bytes) {
    const int T = m.rows >> 3;
    const int P = min(ncta, T);
    Share s;
    if (cta < P) {
        s.a = split_at(T, cta, P);
        s.b = split_at(T, cta + 1, P);
    } else {
        s.a = s.b = 0;
    }
    s.per = max(1, min(kConsThreads / 8, slot_bytes / m.tile_bytes));
    return s;
}

// --------------------------------------------------------- smem layout --

struct DecSmem {
    uint64_t *full;          // ring mbarriers (one per slot)
    struct Feed *feed;       // the feeder thread's cursor
    FeedUnit *plan;          // the CTA's units of one token
    ShareTab *st;            // the CTA's shares (computed at launch)
    Layer *lay;              // descriptors of the current and the next two layers (buffer g % 3, g = layers so far)
    uint8_t *ring;           // nslots * slot_bytes
    float *xv;               // activation vector, paired layout for Q4 / plain for Q8 (max(E,F) floats)
    float *xq8;              // the same vector in plain layout when a Q8_0 matrix reads it
    float *xs;               // raw residual (E floats)
    double *part;            // [kCons][8 tiles-in-unit max 8][8 rows] partial sums
    float *rows;             // row results of a unit [64]
    float *gate;             // gate rows of this CTA's gate/up share (max 8 * 64 rows)
    float *red;              // reduction scratch [64]
    float *att;              // attention scratch
    float *merge;            // attention partials of up to 8 chunks: pv [8][E], then (max, sum) [8][H]
    float *pre;              // the QKV epilogue's bias and RoPE (cos, sin) per row of the CTA's share
    float *kvs;              // an attention item's history K rows, then V rows (aliases xv..gate)
    float *nrm;              // the next norm's weights (embd floats)
};

__device__ __forceinline__ Share share_of(const DecSmem &sm, int kind, const QMat &m) {
    return Share{sm.st->a[kind], sm.st->b[kind], sm.st->per[kind][fmt_ix(m.type)]};
}

// --------------------------------------------------------- dot products --
// The activation vector is staged block by block with a stride of kXB floats
// per 32-wide block (32 values + 4 of padding), so that 8 lanes reading 8
// different blocks hit 8 different bank groups.
constexpr int kXB = 36;

// A tile of 8 rows in shared memory; lane (r, q) = (lane / 4, lane % 4).
// Returns the lane's partial over blocks [b0, b1).  Everything here is on
// the latency-critical path of a phase, so it stays in f32: double
// conversions and FMAs cost hundreds of cycles of latency per block here.

// Q4_0 / Q4_1 with the activation in paired layout: for block b, pair j
// (0..15) = (x[32b + j], x[32b + 16 + j]), so lane q reads pairs 4q..4q+3.
template <bool Q41>
__device__ __forceinline__ float dot_q4(const uint8_t *tile, int nb, const float2 *xp, int b0, int b1, int lane) {
    const int r = lane >> 2, q = lane & 3;
    const uint32_t qw = smem_u32(tile) + 4 * (r * 4 + q);          // + 128 b: this lane's 4 quant bytes of block b
    const uint32_t dp = smem_u32(tile) + nb * 128 + 2 * r;         // + 16 b: the row's scale
    const uint32_t mp = dp + nb * 16;                              // + 16 b: the row's minimum (Q4_1)
    const uint32_t xa0 = smem_u32(xp) + 4 * (8 * q);               // + 4 kXB b: pairs 4q..4q+3 of block b
    const float off = Q41 ? 8388608.f : 8388616.f;
    const float2 off2 = make_float2(off, off);
    float acc = 0.f;
#pragma unroll 4
    for (int b = b0; b < b1; ++b) {
        const uint32_t w = lds_u32(qw + 128 * b);
        const float d = lds_h2f(dp + 16 * b);
        const float4 xa = lds_f4(xa0 + 4 * kXB * b);
        const float4 xb = lds_f4(xa0 + 4 * kXB * b + 16);
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        float2 s = __fmul2_rn(__fadd2_rn(make_float2(b2f(lo, 0), b2f(hi, 0)), make_float2(-off2.x, -off2.y)),
                              make_float2(xa.x, xa.y));
        s = __ffma2_rn(__fadd2_rn(make_float2(b2f(lo, 1), b2f(hi, 1)), make_float2(-off, -off)),
                       make_float2(xa.z, xa.w), s);
        s = __ffma2_rn(__fadd2_rn(make_float2(b2f(lo, 2), b2f(hi, 2)), make_float2(-off, -off)),
                       make_float2(xb.x, xb.y), s);
        s = __ffma2_rn(__fadd2_rn(make_float2(b2f(lo, 3), b2f(hi, 3)), make_float2(-off, -off)),
                       make_float2(xb.z, xb.w), s);
        const float sum = s.x + s.y;
        if (Q41) {
            const float mn = lds_h2f(mp + 16 * b);
            const float2 sx2 = __fadd2_rn(__fadd2_rn(make_float2(xa.x, xa.y), make_float2(xa.z, xa.w)),
                                          __fadd2_rn(make_float2(xb.x, xb.y), make_float2(xb.z, xb.w)));
            acc = fmaf(d, sum, fmaf(mn, sx2.x + sx2.y, acc));
        } else {
            acc = fmaf(d, sum, acc);
        }
    }
    return acc;
}

// Q8_0 with the activation in plain layout: lane q owns elements 8q..8q+7.
__device__ __forceinline__ float dot_q8(const uint8_t *tile, int nb, const float *x, int b0, int b1, int lane) {
    const int r = lane >> 2, q = lane & 3;
    const uint32_t qw = smem_u32(tile) + 8 * (r * 4 + q);          // + 256 b
    const uint32_t dp = smem_u32(tile) + nb * 256 + 2 * r;         // + 16 b
    const uint32_t xa0 = smem_u32(x) + 4 * (8 * q);                // + 4 kXB b
    constexpr float off = 8388736.f;
    float acc = 0.f;
#pragma unroll 4
    for (int b = b0; b < b1; ++b) {
        const uint2 w = lds_u64(qw + 256 * b);
        const float d = lds_h2f(dp + 16 * b);
        const float4 xa = lds_f4(xa0 + 4 * kXB * b);
        const float4 xb = lds_f4(xa0 + 4 * kXB * b + 16);
        const uint32_t u0 = w.x ^ 0x80808080u, u1 = w.y ^ 0x80808080u;
        const float2 o2 = make_float2(-off, -off);
        float2 s = __fmul2_rn(__fadd2_rn(make_float2(b2f(u0, 0), b2f(u0, 1)), o2), make_float2(xa.x, xa.y));
        s = __ffma2_rn(__fadd2_rn(make_float2(b2f(u0, 2), b2f(u0, 3)), o2), make_float2(xa.z, xa.w), s);
        s = __ffma2_rn(__fadd2_rn(make_float2(b2f(u1, 0), b2f(u1, 1)), o2), make_float2(xb.x, xb.y), s);
        s = __ffma2_rn(__fadd2_rn(make_float2(b2f(u1, 2), b2f(u1, 3)), o2), make_float2(xb.z, xb.w), s);
        acc = fmaf(d, s.x + s.y, acc);
    }
    return acc;
}

__device__ __forceinline__ float dot_tile(int type, const uint8_t *tile, int nb, const DecSmem &sm, int b0, int b1,
                                           int lane) {
    if (type == 8) return dot_q8(tile, nb, sm.xq8, b0, b1, lane);
    if (type == 3) return dot_q4<true>(tile, nb, reinterpret_cast<const float2 *>(sm.xv), b0, b1, lane);
    return dot_q4<false>(tile, nb, reinterpret_cast<const float2 *>(sm.xv), b0, b1, lane);
}

// Row r of a tile, one block per lane (lanes b, b + 32, ... of the nb
// blocks), summed over the warp: every lane returns the row's value.  Used
// for units of fewer tiles than warps, where each warp takes whole rows and
// no partial sums cross warps.
__device__ __forceinline__ float dot_row(int type, const uint8_t *tile, int nb, int r, const DecSmem &sm, int lane,
                                         int b0 = 0, int b1 = -1) {
    if (b1 < 0) b1 = nb;
    float acc = 0.f;
    const uint32_t ts = smem_u32(tile);
    if (type == 8) {
        const uint32_t dp = ts + nb * 256 + 2 * r, x0 = smem_u32(sm.xq8);
        for (int b = b0 + lane; b < b1; b += 32) {
            const uint32_t qp = ts + (b * 8 + r) * 32, xp = x0 + 4 * kXB * b;
            const float d = lds_h2f(dp + 16 * b);
            const float2 o2 = make_float2(-8388736.f, -8388736.f);
            float2 s = make_float2(0.f, 0.f);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float4 qf = lds_f4(qp + 16 * h);
                const uint32_t u[4] = {__float_as_uint(qf.x) ^ 0x80808080u, __float_as_uint(qf.y) ^ 0x80808080u,
                                       __float_as_uint(qf.z) ^ 0x80808080u, __float_as_uint(qf.w) ^ 0x80808080u};
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const float4 x = lds_f4(xp + 16 * (4 * h + w));
                    s = __ffma2_rn(__fadd2_rn(make_float2(b2f(u[w], 0), b2f(u[w], 1)), o2), make_float2(x.x, x.y), s);
                    s = __ffma2_rn(__fadd2_rn(make_float2(b2f(u[w], 2), b2f(u[w], 3)), o2), make_float2(x.z, x.w), s);
                }
            }
            acc = fmaf(d, s.x + s.y, acc);
        }
    } else {
        const uint32_t dp = ts + nb * 128 + 2 * r, x0 = smem_u32(sm.xv);
        const float off = type == 3 ? 8388608.f : 8388616.f;
        const float2 o2 = make_float2(-off, -off);
        for (int b = b0 + lane; b < b1; b += 32) {
            const float4 qf = lds_f4(ts + (b * 8 + r) * 16);
            const uint32_t xp = x0 + 4 * kXB * b;  // pairs (x_j, x_j+16)
            const float d = lds_h2f(dp + 16 * b);
            const uint32_t wq[4] = {__float_as_uint(qf.x), __float_as_uint(qf.y), __float_as_uint(qf.z),
                                    __float_as_uint(qf.w)};
            float2 s = make_float2(0.f, 0.f), sx = make_float2(0.f, 0.f);
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const uint32_t lo = wq[w] & 0x0F0F0F0Fu, hi = (wq[w] >> 4) & 0x0F0F0F0Fu;
                const float4 xa = lds_f4(xp + 32 * w), xb = lds_f4(xp + 32 * w + 16);
                s = __ffma2_rn(__fadd2_rn(make_float2(b2f(lo, 0), b2f(hi, 0)), o2), make_float2(xa.x, xa.y), s);
                s = __ffma2_rn(__fadd2_rn(make_float2(b2f(lo, 1), b2f(hi, 1)), o2), make_float2(xa.z, xa.w), s);
                s = __ffma2_rn(__fadd2_rn(make_float2(b2f(lo, 2), b2f(hi, 2)), o2), make_float2(xb.x, xb.y), s);
                s = __ffma2_rn(__fadd2_rn(make_float2(b2f(lo, 3), b2f(hi, 3)), o2), make_float2(xb.z, xb.w), s);
                if (type == 3)
                    sx = __fadd2_rn(sx, __fadd2_rn(__fadd2_rn(make_float2(xa.x, xa.y), make_float2(xa.z, xa.w)),
                                                   __fadd2_rn(make_float2(xb.x, xb.y), make_float2(xb.z, xb.w))));
            }
            if (type == 3) acc = fmaf(d, s.x + s.y, fmaf(lds_h2f(dp + nb * 16 + 16 * b), sx.x + sx.y, acc));
            else acc = fmaf(d, s.x + s.y, acc);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
    return acc;
}

// ------------------------------------------------------------- staging --
// Asynchronous global -> shared copies (cp.async): the issuing thread does not
// wait for them; cp_async_wait_all waits for all of the thread's copies.
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}

// Norm weights into sm.nrm (embd is a multiple of 32, the weights 256-byte
// aligned), issued at the start of the phase before the one that uses them:
// the copies complete while that phase runs, off the path from the input's
// arrival to the first dot product.  norm_fold waits for them.
// cp.async copies complete in no fixed order, so the thread's earlier copies
// (an earlier norm's, into the same bytes) are waited for first; normally
// they are long done.
__device__ __forceinline__ void prefetch_norm(const float *w, int E, const DecSmem &sm) {
    cp_async_wait_all();
    for (int i = threadIdx.x; 4 * i < E; i += kConsThreads) cp_async16(sm.nrm + 4 * i, w + 4 * i);
}

// RMSNorm (cpu.go:81-98), folded: stages x * w (into the layouts the dot
// products read) and leaves the warps' partial sums of squares in red[32..39];
// the scalar 1 / rms (norm_scale) multiplies the dot products' results
// instead of every element, which keeps the sum of squares, the division and
// the square root off the path to the first dot product.  (x * w) * s and
// cpu.go's (x * s) * w differ only in rounding.
__device__ __forceinline__ void norm_fold(const DecParams &dm, const DecSmem &sm, bool q8) {
    const int E = dm.embd;
    cp_async_wait_all();  // this thread's prefetches (norm weights, QKV epilogue inputs), then everyone's
    cons_sync();
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = threadIdx.x + k * kConsThreads;
        if (i >= E) break;
        const float x = sm.xs[i];
        ss = fmaf(x, x, ss);
        const float v = __fmul_rn(x, sm.nrm[i]);
        const int b = i >> 5, j = i & 31, pj = j & 15;
        sm.xv[b * kXB + 2 * pj + (j >> 4)] = v;
        if (q8) sm.xq8[b * kXB + j] = v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
    if ((threadIdx.x & 31) == 0) sm.red[32 + (threadIdx.x >> 5)] = ss;
    cons_sync();
}

// The input poll of a normed phase, fused with norm_fold's staging: each
// thread stages x * w of its word pairs into the dot products' layouts as
// they arrive (round-based, as poll_segs) and returns its sum of squares
// (negative on a device error).  The norm weights must be visible (waited
// for and behind a barrier) before the call.
__device__ __noinline__ float poll_stage(const uint64_t *src, int n, uint32_t tag, float *xv, float *xq8,
                                         const float *nrm, int *err) {
    const int npairs = n >> 1;
    constexpr int K = 4;
    float ss = 0.f;
    for (int base = 0; base < npairs; base += K * kConsThreads) {
        uint64_t v[2 * K];
        unsigned pend = 0;
#pragma unroll
        for (int k = 0; k < K; ++k)
            if (base + threadIdx.x + k * kConsThreads < npairs) pend |= 1u << k;
        const uint64_t t0 = gtimer();
        unsigned spins = 0;
        while (pend) {
#pragma unroll
            for (int k = 0; k < K; ++k)
                if (pend >> k & 1) ld_relaxed2(src + 2 * (base + threadIdx.x + k * kConsThreads), v[2 * k], v[2 * k + 1]);
#pragma unroll
            for (int k = 0; k < K; ++k) {
                if (!(pend >> k & 1)) continue;
                if ((uint32_t)(v[2 * k] >> 32) == tag && (uint32_t)(v[2 * k + 1] >> 32) == tag) {
                    const int i = 2 * (base + threadIdx.x + k * kConsThreads);
                    const float x0 = __uint_as_float((uint32_t)v[2 * k]), x1 = __uint_as_float((uint32_t)v[2 * k + 1]);
                    ss = fmaf(x1, x1, fmaf(x0, x0, ss));
                    const float s0 = __fmul_rn(x0, nrm[i]), s1 = __fmul_rn(x1, nrm[i + 1]);
                    const int b = i >> 5, j = i & 31;  // j even: j and j + 1 in the same block
                    xv[b * kXB + 2 * (j & 15) + (j >> 4)] = s0;
                    xv[b * kXB + 2 * ((j + 1) & 15) + ((j + 1) >> 4)] = s1;
                    if (xq8) xq8[b * kXB + j] = s0, xq8[b * kXB + j + 1] = s1;
                    pend &= ~(1u << k);
                }
            }
            if (pend && (++spins & 255) == 0) {
                if (read_err(err)) return -1.f;
                if (gtimer() - t0 > s_wait_ns) {
                    atomicExch(err, DEV_TAG_TIMEOUT);
                    return -1.f;
                }
            }
        }
    }
    return ss;
}

// The input poll of the output and down phases, fused with the staging:
// word pairs of src0 (n0 values, tag0) are written as they arrive into the
// dot products' layouts (xv, and xq8 unless null), those of src1 (n1 values,
// tag1: the CTA's residual rows) into dst1.  Round-based, as poll_segs.
__device__ __noinline__ bool poll_stage_res(const uint64_t *src0, int n0, uint32_t tag0, float *xv, float *xq8,
                                            const uint64_t *src1, int n1, uint32_t tag1, float *dst1, int *err) {
    const int np0 = n0 >> 1, npairs = np0 + (n1 >> 1);
    constexpr int K = 4;
    for (int base = 0; base < npairs; base += K * kConsThreads) {
        uint64_t v[2 * K];
        unsigned pend = 0;
#pragma unroll
        for (int k = 0; k < K; ++k)
            if (base + threadIdx.x + k * kConsThreads < npairs) pend |= 1u << k;
        const uint64_t t0 = gtimer();
        unsigned spins = 0;
        while (pend) {
#pragma unroll
            for (int k = 0; k < K; ++k) {
                if (!(pend >> k & 1)) continue;
                const int pi = base + threadIdx.x + k * kConsThreads;
                ld_relaxed2(pi < np0 ? src0 + 2 * pi : src1 + 2 * (pi - np0), v[2 * k], v[2 * k + 1]);
            }
#pragma unroll
            for (int k = 0; k < K; ++k) {
                if (!(pend >> k & 1)) continue;
                const int pi = base + threadIdx.x + k * kConsThreads;
                const uint32_t tag = pi < np0 ? tag0 : tag1;
                if ((uint32_t)(v[2 * k] >> 32) != tag || (uint32_t)(v[2 * k + 1] >> 32) != tag) continue;
                const float x0 = __uint_as_float((uint32_t)v[2 * k]), x1 = __uint_as_float((uint32_t)v[2 * k + 1]);
                if (pi < np0) {
                    const int i = 2 * pi, b = i >> 5, j = i & 31;  // j even: j and j + 1 in the same block
                    xv[b * kXB + 2 * (j & 15) + (j >> 4)] = x0;
                    xv[b * kXB + 2 * ((j + 1) & 15) + ((j + 1) >> 4)] = x1;
                    if (xq8) xq8[b * kXB + j] = x0, xq8[b * kXB + j + 1] = x1;
                } else {
                    dst1[2 * (pi - np0)] = x0, dst1[2 * (pi - np0) + 1] = x1;
                }
                pend &= ~(1u << k);
            }
            if (pend && (++spins & 255) == 0) {
                if (read_err(err)) return false;
                if (gtimer() - t0 > s_wait_ns) {
                    atomicExch(err, DEV_TAG_TIMEOUT);
                    return false;
                }
            }
        }
    }
    return true;
}

// The warps' partial sums of squares into red[32..39] (norm_scale reads them).
// (No barrier: the next consumer barrier publishes them.)
__device__ __forceinline__ void norm_partial(float ss, const DecSmem &sm) {
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
    if ((threadIdx.x & 31) == 0) sm.red[32 + (threadIdx.x >> 5)] = ss;
}

// 1 / sqrt(mean of squares + eps), from the warps' partials (fixed order):
// cpu.go:94 rounds 1/sqrt computed in double to float.  Here a float seed
// (rsqrtf, within 2 ulp) and one Newton step in double (error ~1e-13
// relative), rounded to float: the same float but where the exact value is
// within ~1e-13 of a rounding boundary.  Much shorter than a double rsqrt.
__device__ __forceinline__ float norm_scale(const DecParams &dm, const DecSmem &sm) {
    float ss = 0.f;
#pragma unroll
    for (int w = 0; w < kCons; ++w) ss += sm.red[32 + w];
    const float t = __fadd_rn(__fdiv_rn(ss, (float)dm.embd), dm.eps);
    const double y = (double)rsqrtf(t), td = (double)t;
    return (float)(y * fma(-0.5 * td, y * y, 1.5));
}

// ------------------------------------------------------------- consume --
// The consumer side of the ring: waits for the next unit's slot.

struct Ring {
    int nslots, slot_bytes;
    unsigned u;   // units consumed so far
    int sl;       // u % nslots
    unsigned ph;  // (u / nslots) & 1: the parity of the slot's fill
    __device__ __forceinline__ void next() {
        ++u;
        if (++sl == nslots) sl = 0, ph ^= 1u;
    }
};

// The shared-memory views the tile pipeline needs (by value, so the
// out-of-line unit_rows below takes no reference to kernel parameters).
struct UnitCtx {
    uint64_t *full;
    uint8_t *ring;
    float *xv, *xq8, *part, *rows;
};

// This thread's wait for a ring slot's fill (false: timed out or a device
// error; the caller's consumer barrier makes the outcome uniform).
__device__ __forceinline__ bool slot_wait(uint64_t *full, int sl, unsigned ph, int *err) {
    if (mbar_try_wait(full + sl, ph)) return true;
    const uint64_t w0 = clock64(), t0 = gtimer();
    bool ok = true;
    while (!mbar_try_wait(full + sl, ph)) {
        if (read_err(err)) {
            ok = false;
            break;
        }
        if (gtimer() - t0 > s_wait_ns) {
            atomicExch(err, DEV_RING_TIMEOUT);
            ok = false;
            break;
        }
    }
    if (threadIdx.x == 0) s_ring_wait += clock64() - w0;
    return ok;
}

// Computes the rows of one unit (k tiles of matrix m) into c.rows[k * 8]
// (row i of the unit).  All consumer warps take part: with k >= 8 each warp
// takes whole tiles; with k == 1 warp w takes row w, a block per lane;
// otherwise every tile's blocks are split across the warps, whose partials
// meet through shared memory and three shuffles, in a fixed order.  (Measured
// against a split of the unit's tile-blocks into 8 contiguous ranges, which
// keeps all warps busy for 3 and 5-7 tiles: that was 1-3 % slower on both
// benchmark shapes.)
// waited: the caller has waited for the slot and passed a consumer barrier since.
__device__ __forceinline__ bool unit_rows_nl(const QMat &m, const int k, const UnitCtx &c, const int sl,
                                             const unsigned ph, const int slot_bytes, int *err, bool waited) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (!waited && cons_or(!slot_wait(c.full, sl, ph, err))) return false;
    const uint8_t *slot = c.ring + (size_t)sl * slot_bytes;
    DecSmem sm;
    sm.xv = c.xv, sm.xq8 = c.xq8;
    if (k >= kCons) {
        for (int i = warp; i < k; i += kCons) {
            float a = dot_tile(m.type, slot + (size_t)i * m.tile_bytes, m.nb, sm, 0, m.nb, lane);
            a += __shfl_xor_sync(kFull, a, 1);
            a += __shfl_xor_sync(kFull, a, 2);
            if ((lane & 3) == 0) c.rows[i * 8 + (lane >> 2)] = a;
        }
        __syncwarp();
    } else if (k == 1) {
        // one tile: warp w takes its row w, one block per lane, no partial sums across warps
        const float a = dot_row(m.type, slot, m.nb, warp, sm, lane);
        if (lane == 0) c.rows[warp] = a;
    } else {
        const int lg = k == 2 ? 2 : k <= 4 ? 1 : 0;  // parts = kCons / k = 1 << lg (k in 2..7), by shifts
        const int parts = 1 << lg;
        const int tile = warp >> lg, part = warp & (parts - 1);
        float a = 0.f;
        if (tile < k) {
            const int b0 = (m.nb * part) >> lg, b1 = (m.nb * (part + 1)) >> lg;
            a = dot_tile(m.type, slot + (size_t)tile * m.tile_bytes, m.nb, sm, b0, b1, lane);
        }
        __syncwarp();
        a += __shfl_xor_sync(kFull, a, 1);
        a += __shfl_xor_sync(kFull, a, 2);
        // partial of (row r, warp w) -> part[r * 8 + w]: the 8 parts of a row are 8 consecutive lanes
        if ((lane & 3) == 0) c.part[(lane >> 2) * 8 + warp] = a;
        cons_sync();
        if (threadIdx.x < 64) {
            // thread (r, w) = (t / 8, t % 8); warps w = tile * parts + p
            float v = c.part[threadIdx.x];
            const int w = threadIdx.x & 7;
            // sum over p within each tile's group of `parts` consecutive warps
            if (parts >= 2) v += __shfl_xor_sync(kFull, v, 1);
            if (parts >= 4) v += __shfl_xor_sync(kFull, v, 2);
            if (parts >= 8) v += __shfl_xor_sync(kFull, v, 4);
            if ((w & (parts - 1)) == 0 && (w >> lg) < k) c.rows[(w >> lg) * 8 + (threadIdx.x >> 3)] = v;
        }
    }
    cons_sync();
    return true;
}

__device__ __forceinline__ void feed_issue(const DecSmem &sm, int nslots, int slot_bytes);

// One unit: its rows into sm.rows; then the feeder refills the slot it used.
__device__ __forceinline__ bool unit_rows(const DecParams &dm, const QMat &m, int k, const DecSmem &sm, Ring &rg,
                                          bool waited = false) {
    const UnitCtx c{sm.full, sm.ring, sm.xv, sm.xq8, reinterpret_cast<float *>(sm.part), sm.rows};
    const bool ok = unit_rows_nl(m, k, c, rg.sl, rg.ph, rg.slot_bytes, dm.err, waited);
    rg.next();
    if (ok && threadIdx.x == kFeeder) feed_issue(sm, rg.nslots, rg.slot_bytes);
    return ok;
}

// ---------------------------------------------------------------- tags --

__device__ __forceinline__ uint32_t tag_of(uint32_t epoch, int layers, int l, int ph) {
    // ph: 0 QKV, 1 attention, 2 output projection, 3 gate/up, 4 down; l = -1: the embedding
    return epoch * (uint32_t)(8 * (layers + 1)) + (uint32_t)(8 * (l + 1) + ph) + 1u;
}

enum { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_HEAD = 5 };

// Gate and up tiles of a CTA travel as one unit when they have one format and
// fit one slot (the feeder copies both ranges into the slot).
__device__ __forceinline__ bool gu_fused(const Layer &L, const Share &sg, int slot_bytes) {
    const int n = sg.b - sg.a;
    return L.gate.type == L.up.type && L.gate.nb == L.up.nb && 2 * n * L.gate.tile_bytes <= slot_bytes &&
           2 * n <= kConsThreads / 8;
}

// ------------------------------------------------------------- feeding --
// The weight ring is filled by one consumer thread (kFeeder).  It issues the
// CTA's units in the order the phases consume them: per token and layer the
// QKV tiles one at a time, the output projection's share, gate and up (one
// unit of two copies when gu_fused, else gate's share, then up's), down's
// share; after the last layer the head's share.  A slot is refilled as soon
// as the consumers have finished the unit in it, so the copies run nslots
// units ahead of the consumers.  The sequence is the same for every token;
// k_feed_plan lists it once per model (feed_next below), and the decode
// kernel keeps the CTA's list in shared memory, so a refill is a few
// instructions on the consumers' path.

struct Feed {
    int i, l, st, t;  // planning: token, layer, stage (0 QKV, 1 O, 2 gate or gate+up, 3 up, 4 down, 5 head), cursor
    unsigned issued;  // units issued
    int j, n;         // decoding: the next plan entry, entries per token
    unsigned total;   // units of the launch
    int sl;           // the slot of the next issue (issued % nslots)
};
static_assert(sizeof(Feed) <= 64, "the shared-memory layout reserves 64 bytes");

__device__ __forceinline__ bool share_unit(const QMat &m, const Share &s, int &ft, const uint8_t *&src, unsigned &n) {
    const int t = s.a + ft;
    if (t >= s.b) return false;
    src = m.tiles + (size_t)t * m.tile_bytes;
    n = (unsigned)(min(s.per, s.b - t) * m.tile_bytes);
    ft += s.per;
    return true;
}

// The next unit's one or two source ranges; false once the sequence is done.
__device__ bool feed_next(const DecParams &dm, Feed &f, int ntok, int slot_bytes, const uint8_t *&s1, unsigned &n1,
                          const uint8_t *&s2, unsigned &n2) {
    const int cta = blockIdx.x, ncta = gridDim.x;
    n2 = 0;
    while (f.i < ntok) {
        if (f.st == 5) {
            if (share_unit(dm.head, share(dm.head, cta, ncta, slot_bytes), f.t, s1, n1)) return true;
            f.i++, f.l = 0, f.st = 0, f.t = 0;
            continue;
        }
        const Layer &L = dm.layer[f.l];
        if (f.st == 0) {
            const int nq = L.q.rows >> 3, nk = L.k.rows >> 3, T = nq + nk + (L.v.rows >> 3);
            const int P = dec_qkv_ctas(T, ncta, dm.heads);
            if (cta < P) {
                const int a = split_at(T, cta, P), b = split_at(T, cta + 1, P);
                const int t = a + f.t;
                if (t < b) {
                    const QMat &m = t < nq ? L.q : t < nq + nk ? L.k : L.v;
                    const int lt = t < nq ? t : t < nq + nk ? t - nq : t - nq - nk;
                    s1 = m.tiles + (size_t)lt * m.tile_bytes;
                    n1 = (unsigned)m.tile_bytes;
                    f.t++;
                    return true;
                }
            }
        } else if (f.st == 2) {
            const Share sg = share(L.gate, cta, ncta, slot_bytes);
            if (sg.b > sg.a && gu_fused(L, sg, slot_bytes)) {
                if (f.t == 0) {
                    n1 = n2 = (unsigned)((sg.b - sg.a) * L.gate.tile_bytes);
                    s1 = L.gate.tiles + (size_t)sg.a * L.gate.tile_bytes;
                    s2 = L.up.tiles + (size_t)sg.a * L.up.tile_bytes;
                    f.t = 1;
                    return true;
                }
                f.st = 4, f.t = 0;  // up travelled with gate
                continue;
            }
            if (share_unit(L.gate, sg, f.t, s1, n1)) return true;
        } else if (f.st == 4 && down_halves(L.down, ncta)) {
            if (f.t == 0 && cta < 2 * (L.down.rows >> 3)) {  // half tile cta: the whole tile travels
                s1 = L.down.tiles + (size_t)(cta >> 1) * L.down.tile_bytes;
                n1 = (unsigned)L.down.tile_bytes;
                f.t = 1;
                return true;
            }
        } else {
            const QMat &m = f.st == 1 ? L.o : f.st == 3 ? L.up : L.down;
            if (share_unit(m, share(m, cta, ncta, slot_bytes), f.t, s1, n1)) return true;
        }
        f.t = 0;
        if (f.st < 4) f.st++;
        else if (f.l + 1 < dm.layers) f.l++, f.st = 0;
        else f.st = 5;
    }
    return false;
}

// Issues the next unit into the slot that follows the last one issued (the
// caller guarantees the consumers are done with that slot).
__device__ __forceinline__ void feed_issue(const DecSmem &sm, int nslots, int slot_bytes) {
    Feed &f = *sm.feed;
    if (f.issued >= f.total) return;
    const FeedUnit e = sm.plan[f.j];
    f.j = f.j + 1 == f.n ? 0 : f.j + 1;
    const int slot = f.sl;
    f.sl = f.sl + 1 == nslots ? 0 : f.sl + 1;
    uint8_t *dst = sm.ring + (size_t)slot * slot_bytes;
    // the slot's previous contents were read through the generic proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(sm.full + slot, e.n1 + e.n2);
    bulk_g2s(dst, e.src1, e.n1, sm.full + slot);
    if (e.n2) bulk_g2s(dst + e.n1, e.src2, e.n2, sm.full + slot);
    f.issued++;
}

// Lists each CTA's units of one token (one thread per CTA, the decode
// kernel's grid); count -1 if they exceed kMaxFeedPlan.
__global__ void k_feed_plan(const __grid_constant__ DecParams dm, int slot_bytes, FeedUnit *plan, int *count) {
    if (threadIdx.x != 0) return;
    Feed f{};
    FeedUnit *out = plan + (size_t)blockIdx.x * kMaxFeedPlan;
    const uint8_t *s1, *s2;
    unsigned n1, n2;
    int n = 0;
    while (feed_next(dm, f, 1, slot_bytes, s1, n1, s2, n2)) {
        if (n == kMaxFeedPlan) {
            count[blockIdx.x] = -1;
            return;
        }
        out[n++] = FeedUnit{s1, n2 ? s2 : nullptr, n1, n2};
    }
    count[blockIdx.x] = n;
}

// Before the CTA exits: waits (bounded) for the copies issued but not consumed
// (only an error path leaves any).
__device__ void feed_drain(const DecSmem &sm, int nslots, unsigned consumed) {
    for (unsigned v = consumed; v < sm.feed->issued; ++v) {
        const uint64_t t0 = gtimer();
        while (!mbar_try_wait(sm.full + v % nslots, (v / nslots) & 1))
            if (gtimer() - t0 > s_wait_ns / 4) break;
    }
}

// -------------------------------------------------------------- phases --

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

struct Tok {
    int pos, step, tok;
    uint32_t epoch;
    int g0;    // layers of the launch before this token's (indexes the descriptor buffers)
    Trace tr;  // this token's timeline (first token of a launch only)
};

// Per-layer descriptors are read from shared memory rather than from the
// kernel parameter's constant bank (measured a little faster).  Layer
// g % layers of the launch's sequence goes to buffer g % 3, copied two layers
// ahead (cp.async) and waited for at the top of the layer before it.
__device__ __forceinline__ const Layer &lay(const DecSmem &sm, const Tok &tk, int l) { return sm.lay[(tk.g0 + l) % 3]; }

__device__ __forceinline__ void fetch_layer(const DecParams &dm, const DecSmem &sm, int g) {
    constexpr int NP = (int)(sizeof(Layer) / 16);
    if (threadIdx.x < NP)
        cp_async16(reinterpret_cast<char *>(sm.lay + g % 3) + 16 * threadIdx.x,
                   reinterpret_cast<const char *>(dm.layers_g + g % dm.layers) + 16 * threadIdx.x);
}

// K1: RMSNorm + QKV + bias + RoPE + KV append (kernels_fused.go:47-73).
// The QKV epilogue's inputs that do not depend on the token's activations
// (bias, RoPE cos and sin of the position), and the attention norm's weights:
// issued before the previous layer's down projection.
__device__ __forceinline__ void qkv_prefetch(const DecParams &dm, int l, const Tok &tk, const DecSmem &sm) {
    const Layer &L = lay(sm, tk, l);
    const int a = sm.st->a[SK_QKV], b = sm.st->b[SK_QKV];
    if (b <= a) return;
    const int nq = L.q.rows >> 3, nk = L.k.rows >> 3;
    prefetch_norm(L.attn_norm, dm.embd, sm);
    const int hp = dm.head_dim >> 1;
    for (int i = threadIdx.x; i < (b - a) * 8; i += kConsThreads) {
        const int t = a + (i >> 3), r = i & 7;
        const int seg = t < nq ? 0 : t < nq + nk ? 1 : 2;
        const int row = (seg == 0 ? t : seg == 1 ? t - nq : t - nq - nk) * 8 + r;
        const float *bias = seg == 0 ? L.bq : seg == 1 ? L.bk : L.bv;
        if (bias) cp_async4(sm.pre + 4 * i, bias + row);
        else sm.pre[4 * i] = 0.f;
        if (seg < 2)
            cp_async8(sm.pre + 4 * i + 2, reinterpret_cast<const float2 *>(dm.rope_cs) + (size_t)tk.pos * hp +
                                              ((row & (dm.head_dim - 1)) >> 1));  // head_dim: 64 or 128
        else
            sm.pre[4 * i + 2] = 1.f, sm.pre[4 * i + 3] = 0.f;
    }
}

__device__ bool ph_qkv(const DecParams &dm, int l, const Tok &tk, const DecSmem &sm, Ring &rg) {
    const Layer &L = lay(sm, tk, l);
    const int a = sm.st->a[SK_QKV], b = sm.st->b[SK_QKV];
    if (b <= a) return true;
    const int nq = L.q.rows >> 3, nk = L.k.rows >> 3;
    const int E = dm.embd, ev = l * 5 + PH_QKV;
    tk.tr.stamp(ev, 0);
    const uint32_t tag_in = tag_of(tk.epoch, dm.layers, l - 1, PH_DOWN);
    if (l == 0) {
        for (int e = threadIdx.x; e < E; e += kConsThreads) {
            const QMat &m = dm.embed;
            const uint8_t *t = m.tiles + (size_t)(tk.tok >> 3) * m.tile_bytes;
            const int r = tk.tok & 7, b = e >> 5, j = e & 31, qb = m.type == 8 ? 32 : 16;
            const float d = __half2float(reinterpret_cast<const __half *>(t + (size_t)m.nb * 8 * qb)[b * 8 + r]);
            const uint8_t *qs = t + ((size_t)b * 8 + r) * qb;
            float v;
            if (m.type == 8) v = d * (float)(int8_t)qs[j];
            else v = d * (float)(((j < 16) ? (qs[j & 15] & 15) : (qs[j & 15] >> 4)) - 8);
            sm.xs[e] = v;
        }
        cons_sync();
    }
    const bool q8 = L.q.type == 8 || L.k.type == 8 || L.v.type == 8;
    if (l == 0) {
        tk.tr.stamp(ev, 1);
        norm_fold(dm, sm, q8);
    } else {
        cp_async_wait_all();  // the norm weights, prefetched during the phase before
        cons_sync();
        const float ss = poll_stage(dm.ll_x, E, tag_in, sm.xv, q8 ? sm.xq8 : nullptr, sm.nrm, dm.err);
        norm_partial(ss, sm);
        // one barrier for the activations, the norm partials and the first unit's slot
        if (cons_or(ss < 0.f || !slot_wait(sm.full, rg.sl, rg.ph, dm.err))) return false;
        tk.tr.stamp(ev, 1);
    }
    const float nsc = norm_scale(dm, sm);
    const uint32_t tag = tag_of(tk.epoch, dm.layers, l, PH_QKV);
    for (int t = a; t < b; ++t) {
        const int seg = t < nq ? 0 : t < nq + nk ? 1 : 2;
        const QMat &m = seg == 0 ? L.q : seg == 1 ? L.k : L.v;
        const int lt = seg == 0 ? t : seg == 1 ? t - nq : t - nq - nk;
        if (!unit_rows(dm, m, 1, sm, rg, l > 0 && t == a)) return false;
        if (threadIdx.x < 8) {
            const int r = threadIdx.x, row = lt * 8 + r;
            const float *pre = sm.pre + 4 * ((t - a) * 8);
            const bool has_bias = (seg == 0 ? L.bq : seg == 1 ? L.bk : L.bv) != nullptr;
            float v = __fmul_rn(sm.rows[r], nsc);
            if (has_bias) v = __fadd_rn(v, pre[4 * r]);
            if (seg < 2) {
                float o = __fmul_rn(sm.rows[r ^ 1], nsc);
                if (has_bias) o = __fadd_rn(o, pre[4 * (r ^ 1)]);
                const float2 cs = make_float2(pre[4 * r + 2], pre[4 * r + 3]);
                if ((r & 1) == 0) v = __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(o, cs.y));
                else v = __fadd_rn(__fmul_rn(o, cs.y), __fmul_rn(v, cs.x));
            }
            if (seg == 0) {
                ll_put(dm.ll_q + row, v, tag);
            } else if (seg == 1) {
                L.kv[(size_t)tk.pos * dm.kvd + row] = v;
                ll_put(dm.ll_k + row, v, tag);
            } else {
                L.kv[((size_t)dm.ctx + tk.pos) * dm.kvd + row] = v;
                ll_put(dm.ll_v + row, v, tag);
            }
        }
        cons_sync();
    }
    tk.tr.stamp(ev, 2);
    return true;
}

// The end of an attention item, after the warps' partials (V sum, max, sum
// of exp) are in wpart and a consumer barrier: their combination, then the
// head's output (one item), the item's partial (several), or, for the item
// holding the current position, the merge of the head's items.
template <int HD>
__device__ __forceinline__ bool attn_finish(const DecParams &dm, const DecSmem &sm, const float *wpart, int h, int c,
                                            int nch, bool has_cur, uint32_t otag) {
    // the warps' partials combined: thread d < HD sums dimension d
    float *own = sm.merge;  // the merging item's own partial: V sum [HD], max, sum of exp
    const int d = threadIdx.x;
    float cm = -FLT_MAX, cl = 0.f, co = 0.f;
    if (d < HD) {
        // a warp without positions left max -FLT_MAX, sum 0 and a zero V sum:
        // its factor is exp(-huge) = 0
        float2 ml[kCons];
        float ow[kCons];
#pragma unroll
        for (int w = 0; w < kCons; ++w) {
            ml[w] = *reinterpret_cast<const float2 *>(wpart + w * (HD + 4) + HD);
            ow[w] = wpart[w * (HD + 4) + d];
        }
#pragma unroll
        for (int w = 0; w < kCons; ++w) cm = fmaxf(cm, ml[w].x);
        float cl1 = 0.f, co1 = 0.f;
#pragma unroll
        for (int w = 0; w < kCons; w += 2) {
            const float f0 = expf(__fsub_rn(ml[w].x, cm)), f1 = expf(__fsub_rn(ml[w + 1].x, cm));
            cl = fmaf(f0, ml[w].y, cl), cl1 = fmaf(f1, ml[w + 1].y, cl1);
            co = fmaf(f0, ow[w], co), co1 = fmaf(f1, ow[w + 1], co1);
        }
        cl += cl1, co += co1;
        const size_t pi = (size_t)h * dm.nchunk + c;  // head-major: a head's chunks are contiguous
        if (nch == 1) ll_put(dm.ll_att + h * HD + d, __fdiv_rn(co, cl), otag);
        else if (has_cur) own[d] = co;
        else ll_put(dm.ll_pv + pi * HD + d, co, otag);
        if (nch > 1 && d == 0) {
            if (has_cur) {
                own[HD] = cm, own[HD + 1] = cl;
            } else {
                ll_put(dm.ll_ml + pi * 2, cm, otag);
                ll_put(dm.ll_ml + pi * 2 + 1, cl, otag);
            }
        }
    }
    if (nch == 1) return true;  // nothing reads the partials' bytes before the next item's own barriers
    cons_sync();
    if (has_cur) {
        // The item holding the current position merges the head's other chunks
        // (kernels_fused.go:150-170) in groups of up to 8, running max and sums
        // in double, and publishes the head's output.
        float *gpv = own + HD + 16, *gml = gpv + 8 * HD;
        const int d = threadIdx.x;
        double M = own[HD], Ls = own[HD + 1], O = d < HD ? (double)own[d] : 0.0;
        for (int c0 = 0; c0 < nch - 1; c0 += 8) {
            const int gn = min(8, nch - 1 - c0);
            const size_t pi = (size_t)h * dm.nchunk + c0;
            if (cons_or(!poll_two(dm.ll_pv + pi * HD, gn * HD, otag, gpv, dm.ll_ml + pi * 2, gn * 2, otag, gml, dm.err)))
                return false;
            if (d < HD) {
                double Mn = M;
                for (int k = 0; k < gn; ++k) Mn = fmax(Mn, (double)gml[2 * k]);
                const double rs = exp(M - Mn);
                O *= rs, Ls *= rs;
                for (int k = 0; k < gn; ++k) {
                    const double f = exp((double)gml[2 * k] - Mn);
                    Ls = fma(f, (double)gml[2 * k + 1], Ls);
                    O = fma(f, (double)gpv[k * HD + d], O);
                }
                M = Mn;
            }
            cons_sync();
        }
        if (d < HD) ll_put(dm.ll_att + h * HD + d, (float)(O / Ls), otag);
    }
    return true;
}


// K2 (head_dim 128; head_dim 64 runs ph_attn_r64 below): attention of the
// token (n = pos + 1 positions) for item (head,
// chunk of dm.dec_chunk positions): scores, max and sum of exp, the
// exp-weighted V sum (kernels_fused.go:82-146).  The chunk's cached K and V
// rows do not depend on this token, so they are copied into shared memory
// (cp.async) before the item waits for the token's q, k, v.  Each warp takes
// a share of the positions (a multiple of 8), a lane per position for the
// scores and a lane per HD/32 dimensions for the V sum, with its own max; the
// eight warp partials are then combined.  With one chunk the item writes the
// head's output; otherwise the item holding the current position merges the
// others' partials.  f32 arithmetic (the exp in double in cpu.go:321: within
// 2 ulp), the merge of chunks in double.
//
// K rows sit at a stride of HD + 4 floats: a quarter warp reading the same
// 16 bytes of 8 consecutive rows touches each bank once.  V rows are read a
// row per warp instruction, at a stride of HD; the current position's V row
// is polled into place, its K row into kc.
template <int HD>
__device__ bool ph_attn_t(const DecParams &dm, int l, const Tok &tk, int item, int nch, const DecSmem &sm) {
    constexpr int KS = HD + 4;
    constexpr int V4 = HD / 4;
    constexpr int VD = HD / 32;  // V dimensions per lane
    const int grp = dm.heads / dm.kv_heads;
    const int h = item / nch, c = item % nch, kvh = h / grp;
    const int n = tk.pos + 1, C = dm.dec_chunk;
    const Layer &L = lay(sm, tk, l);
    const uint32_t tag = tag_of(tk.epoch, dm.layers, l, PH_QKV);
    const uint32_t otag = tag_of(tk.epoch, dm.layers, l, PH_ATT);
    float *qh = sm.att, *kc = sm.att + HD;
    float *wpart = sm.att + 3 * HD;  // [8 warps][HD + 4]: V sum, then max and sum of exp
    float *ks = sm.kvs, *vs = sm.kvs + (size_t)C * KS;
    const int p0 = c * C, cnt = min(C, n - p0);
    const bool has_cur = p0 + cnt == n;
    const int nhist = has_cur ? cnt - 1 : cnt;
    const int ev = l * 5 + PH_ATT;
    tk.tr.stamp(ev, 0);
    cons_sync();  // the K/V rows share their bytes with the previous phase's vectors
    for (int i = threadIdx.x; i < nhist * V4; i += kConsThreads) {
        const int p = i / V4, d4 = i % V4;
        const size_t row = (size_t)(p0 + p) * dm.kvd + kvh * HD + d4 * 4;
        cp_async16(ks + p * KS + d4 * 4, L.kv + row);
        cp_async16(vs + p * HD + d4 * 4, L.kv + (size_t)dm.ctx * dm.kvd + row);
    }
    // V rows past the last position up to a multiple of 8 are read with weight 0: finite
    const int cnt8 = (cnt + 7) & ~7;
    for (int i = cnt * HD + threadIdx.x; i < cnt8 * HD; i += kConsThreads) vs[i] = 0.f;
    const int ncur = has_cur ? HD : 0;
    const Seg qkv[3] = {{dm.ll_q + h * HD, HD, tag, qh}, {dm.ll_k + kvh * HD, ncur, tag, kc},
                        {dm.ll_v + kvh * HD, ncur, tag, vs + nhist * HD}};
    const bool ok = poll_segs(qkv, dm.err);
    cp_async_wait_all();
    if (cons_or(!ok)) return false;
    tk.tr.stamp(ev, 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = ((cnt + kCons - 1) / kCons + 7) & ~7;  // positions per warp: a multiple of 8, at most 32
    const int wp0 = warp * per, wcnt = max(0, min(per, cnt - wp0));
    // scores: a lane per position
    float sc = -FLT_MAX;
    if (lane < wcnt) {
        const int p = wp0 + lane;
        const float *kr = p == nhist ? kc : ks + p * KS;
        float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
#pragma unroll 8
        for (int g = 0; g < V4; ++g) {
            const float4 k4 = *reinterpret_cast<const float4 *>(kr + 4 * g);
            const float4 q4 = *reinterpret_cast<const float4 *>(qh + 4 * g);
            a01 = __ffma2_rn(make_float2(q4.x, q4.y), make_float2(k4.x, k4.y), a01);
            a23 = __ffma2_rn(make_float2(q4.z, q4.w), make_float2(k4.z, k4.w), a23);
        }
        sc = __fmul_rn((a01.x + a01.y) + (a23.x + a23.y), dm.scale);
    }
    float mx = sc;
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    const float e = lane < wcnt ? expf(__fsub_rn(sc, mx)) : 0.f;  // cpu.go:321
    // the V sum, 8 positions at a time, and the sum of exp alongside
    float2 ov[VD / 2];
#pragma unroll
    for (int k = 0; k < VD / 2; ++k) ov[k] = make_float2(0.f, 0.f);
    float ls = 0.f;
    for (int j0 = 0; j0 < wcnt; j0 += 8) {
        const float *vb = vs + (wp0 + j0) * HD + VD * lane;
        float w[8];
        float2 v[8][VD / 2];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            w[k] = __shfl_sync(kFull, e, j0 + k);
            if constexpr (VD == 2) {
                v[k][0] = *reinterpret_cast<const float2 *>(vb + k * HD);
            } else {
                const float4 t = *reinterpret_cast<const float4 *>(vb + k * HD);
                v[k][0] = make_float2(t.x, t.y), v[k][1] = make_float2(t.z, t.w);
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            ls += w[k];
#pragma unroll
            for (int i = 0; i < VD / 2; ++i) ov[i] = __ffma2_rn(make_float2(w[k], w[k]), v[k][i], ov[i]);
        }
    }
    float *wp = wpart + warp * (HD + 4);
#pragma unroll
    for (int k = 0; k < VD / 2; ++k) *reinterpret_cast<float2 *>(wp + VD * lane + 2 * k) = ov[k];
    if (lane == 0) wp[HD] = mx, wp[HD + 1] = ls;
    cons_sync();
    if (!attn_finish<HD>(dm, sm, wpart, h, c, nch, has_cur, otag)) return false;
    tk.tr.stamp(ev, 2);
    return true;
}

// K2 for head_dim 64: the same item with its cached K and V in registers
// instead of shared memory.  At the item's start each lane loads the K row of
// its position (the warp's share is at most 32 positions) and the two V
// columns (2 lane, 2 lane + 1) of every position of the warp's share, from the
// cache through L2; the token's q, k, v are then polled inline (a call would
// spill those registers).  Scores, softmax and the V sum as ph_attn_t, without
// the shared-memory traffic that bounded them.
__device__ bool ph_attn_r64(const DecParams &dm, int l, const Tok &tk, int item, int nch, const DecSmem &sm) {
    constexpr int HD = 64;
    const int grp = dm.heads / dm.kv_heads;
    const int h = item / nch, c = item % nch, kvh = h / grp;
    const int n = tk.pos + 1, C = dm.dec_chunk;
    const Layer &L = lay(sm, tk, l);
    const uint32_t tag = tag_of(tk.epoch, dm.layers, l, PH_QKV);
    const uint32_t otag = tag_of(tk.epoch, dm.layers, l, PH_ATT);
    float *qh = sm.att, *kc = sm.att + HD, *vc = sm.att + 2 * HD;
    float *wpart = sm.att + 3 * HD;  // [8 warps][HD + 4]: V sum, then max and sum of exp
    const int p0 = c * C, cnt = min(C, n - p0);
    const bool has_cur = p0 + cnt == n;
    const int nhist = has_cur ? cnt - 1 : cnt;
    const int ev = l * 5 + PH_ATT;
    tk.tr.stamp(ev, 0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = (cnt + kCons - 1) / kCons;  // positions per warp, at most 32
    const int wp0 = warp * per, wcnt = max(0, min(per, cnt - wp0));
    const float *kb = L.kv + (size_t)p0 * dm.kvd + kvh * HD;
    const float *vb = kb + (size_t)dm.ctx * dm.kvd;
    float4 kr[HD / 4];
    float2 vr[32];
    const int pk = wp0 + lane;
    if (lane < wcnt && pk != nhist) {
        const float4 *src = reinterpret_cast<const float4 *>(kb + (size_t)pk * dm.kvd);
#pragma unroll
        for (int g = 0; g < HD / 4; ++g) kr[g] = ld_cg_early(src + g);
    } else {
#pragma unroll
        for (int g = 0; g < HD / 4; ++g) kr[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j)
        vr[j] = j < wcnt && wp0 + j != nhist
                    ? ld_cg_early(reinterpret_cast<const float2 *>(vb + (size_t)(wp0 + j) * dm.kvd) + lane)
                    : make_float2(0.f, 0.f);
    // q (and k, v when the item holds the current position): a thread per pair of words
    bool ok = true;
    {
        constexpr int NPQ = HD / 2;
        const int np = has_cur ? 3 * NPQ : NPQ, i = threadIdx.x;
        if (i < np) {
            const int sg = i / NPQ, j = i % NPQ;
            const uint64_t *src = (sg == 0 ? dm.ll_q + h * HD : sg == 1 ? dm.ll_k + kvh * HD : dm.ll_v + kvh * HD) + 2 * j;
            float *dst = (sg == 0 ? qh : sg == 1 ? kc : vc) + 2 * j;
            uint64_t a, b;
            ld_relaxed2(src, a, b);
            if ((uint32_t)(a >> 32) != tag || (uint32_t)(b >> 32) != tag) {
                const uint64_t t0 = gtimer();
                unsigned spins = 0;
                while (true) {
                    ld_relaxed2(src, a, b);
                    if ((uint32_t)(a >> 32) == tag && (uint32_t)(b >> 32) == tag) break;
                    if ((++spins & 255) == 0) {
                        if (read_err(dm.err)) {
                            ok = false;
                            break;
                        }
                        if (gtimer() - t0 > s_wait_ns) {
                            atomicExch(dm.err, DEV_TAG_TIMEOUT);
                            ok = false;
                            break;
                        }
                    }
                }
            }
            dst[0] = __uint_as_float((uint32_t)a), dst[1] = __uint_as_float((uint32_t)b);
        }
    }
    if (cons_or(!ok)) return false;
    tk.tr.stamp(ev, 1);
    if (lane < wcnt && pk == nhist) {  // the current position's K row came with the poll
#pragma unroll
        for (int g = 0; g < HD / 4; ++g) kr[g] = *reinterpret_cast<const float4 *>(kc + 4 * g);
    }
    // scores: a lane per position
    float sc = -FLT_MAX;
    if (lane < wcnt) {
        float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
        float2 b01 = make_float2(0.f, 0.f), b23 = make_float2(0.f, 0.f);
#pragma unroll
        for (int g = 0; g < HD / 4; g += 2) {
            const float4 k4 = kr[g], k5 = kr[g + 1];
            const float4 q4 = *reinterpret_cast<const float4 *>(qh + 4 * g);
            const float4 q5 = *reinterpret_cast<const float4 *>(qh + 4 * g + 4);
            a01 = __ffma2_rn(make_float2(q4.x, q4.y), make_float2(k4.x, k4.y), a01);
            a23 = __ffma2_rn(make_float2(q4.z, q4.w), make_float2(k4.z, k4.w), a23);
            b01 = __ffma2_rn(make_float2(q5.x, q5.y), make_float2(k5.x, k5.y), b01);
            b23 = __ffma2_rn(make_float2(q5.z, q5.w), make_float2(k5.z, k5.w), b23);
        }
        sc = __fmul_rn(((a01.x + a01.y) + (a23.x + a23.y)) + ((b01.x + b01.y) + (b23.x + b23.y)), dm.scale);
    }
    float mx = sc;
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    const float e = lane < wcnt ? expf(__fsub_rn(sc, mx)) : 0.f;  // cpu.go:321
    // the V sum over the warp's positions, and the sum of exp alongside: all
    // 32 slots without branches (past the share both the weight and the
    // registers are 0), in two chains; the current position's V column came
    // with the poll and is added last (its weight is in the sum already)
    float2 ov0 = make_float2(0.f, 0.f), ov1 = make_float2(0.f, 0.f);
    float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        const float w0 = __shfl_sync(kFull, e, j), w1 = __shfl_sync(kFull, e, j + 1);
        ov0 = __ffma2_rn(make_float2(w0, w0), vr[j], ov0);
        ov1 = __ffma2_rn(make_float2(w1, w1), vr[j + 1], ov1);
        ls0 += w0, ls1 += w1;
    }
    float2 ov = make_float2(ov0.x + ov1.x, ov0.y + ov1.y);
    float ls = ls0 + ls1;
    const int jc = nhist - wp0;
    if (jc >= 0 && jc < wcnt) {
        const float w = __shfl_sync(kFull, e, jc);
        ov = __ffma2_rn(make_float2(w, w), *reinterpret_cast<const float2 *>(vc + 2 * lane), ov);
    }
    float *wp = wpart + warp * (HD + 4);
    *reinterpret_cast<float2 *>(wp + 2 * lane) = ov;
    if (lane == 0) wp[HD] = mx, wp[HD + 1] = ls;
    cons_sync();
    if (!attn_finish<HD>(dm, sm, wpart, h, c, nch, has_cur, otag)) return false;
    tk.tr.stamp(ev, 2);
    return true;
}

__device__ bool ph_attn(const DecParams &dm, int l, const Tok &tk, int item, int nch, const DecSmem &sm) {
    return dm.head_dim == 128 ? ph_attn_t<128>(dm, l, tk, item, nch, sm) : ph_attn_r64(dm, l, tk, item, nch, sm);
}

// K3: x += Wo att (cpu.go:336-339).
__device__ bool ph_o(const DecParams &dm, int l, const Tok &tk, const DecSmem &sm, Ring &rg) {
    const Layer &L = lay(sm, tk, l);
    const Share s = share_of(sm, SK_O, L.o);
    if (s.b <= s.a) return true;
    const uint32_t tin = tag_of(tk.epoch, dm.layers, l - 1, PH_DOWN);
    const int ev = l * 5 + PH_O;
    tk.tr.stamp(ev, 0);
    const uint32_t tatt = tag_of(tk.epoch, dm.layers, l, PH_ATT);
    if (cons_or(!poll_stage_res(dm.ll_att, dm.embd, tatt, sm.xv, L.o.type == 8 ? sm.xq8 : nullptr,
                                dm.ll_x + s.a * 8, (s.b - s.a) * 8, tin, sm.gate, dm.err) ||
                !slot_wait(sm.full, rg.sl, rg.ph, dm.err)))
        return false;
    tk.tr.stamp(ev, 1);
    const uint32_t tag = tag_of(tk.epoch, dm.layers, l, PH_O);
    for (int t = s.a; t < s.b; t += s.per) {
        const int k = min(s.per, s.b - t);
        if (!unit_rows(dm, L.o, k, sm, rg, t == s.a)) return false;
        // (drop_step: a test aid that makes the next phase's wait run out)
        if (threadIdx.x < k * 8 && !(tk.step == dm.drop_step && l == 0 && blockIdx.x == 0)) {
            const int row = t * 8 + threadIdx.x;
            ll_put(dm.ll_x + row, __fadd_rn(sm.gate[row - s.a * 8], sm.rows[threadIdx.x]), tag);
        }
        cons_sync();
    }
    tk.tr.stamp(ev, 2);
    return true;
}

// K4: RMSNorm + gate/up + SwiGLU (cpu.go:340-346).
__device__ bool ph_gu(const DecParams &dm, int l, const Tok &tk, const DecSmem &sm, Ring &rg) {
    const Layer &L = lay(sm, tk, l);
    const Share sg = share_of(sm, SK_GU, L.gate);
    const Share su = share_of(sm, SK_GU, L.up);
    if (sg.b <= sg.a) return true;
    const int E = dm.embd, ev = l * 5 + PH_GU;
    tk.tr.stamp(ev, 0);
    const uint32_t tin = tag_of(tk.epoch, dm.layers, l, PH_O);
    cp_async_wait_all();  // the norm weights, prefetched during the phase before
    cons_sync();
    const float ss =
        poll_stage(dm.ll_x, E, tin, sm.xv, L.gate.type == 8 || L.up.type == 8 ? sm.xq8 : nullptr, sm.nrm, dm.err);
    norm_partial(ss, sm);
    if (cons_or(ss < 0.f || !slot_wait(sm.full, rg.sl, rg.ph, dm.err))) return false;
    tk.tr.stamp(ev, 1);
    const float nsc = norm_scale(dm, sm);
    const uint32_t tag = tag_of(tk.epoch, dm.layers, l, PH_GU);
    auto swiglu = [&](int row, float g, float u) {
        if (row < dm.ff) {
            // cpu.go:345 rounds exp in double to float; expf is within 2 ulp of that
            const float den = __fadd_rn(1.f, expf(-g));
            ll_put(dm.ll_act + row, __fmul_rn(__fdiv_rn(g, den), u), tag);
        }
    };
    if (gu_fused(L, sg, rg.slot_bytes)) {
        const int n = sg.b - sg.a;
        if (!unit_rows(dm, L.gate, 2 * n, sm, rg, true)) return false;
        if (threadIdx.x < n * 8)
            swiglu(sg.a * 8 + threadIdx.x, __fmul_rn(sm.rows[threadIdx.x], nsc),
                   __fmul_rn(sm.rows[n * 8 + threadIdx.x], nsc));
        cons_sync();
    } else {
        for (int t = sg.a; t < sg.b; t += sg.per) {
            const int k = min(sg.per, sg.b - t);
            if (!unit_rows(dm, L.gate, k, sm, rg, t == sg.a)) return false;
            if (threadIdx.x < k * 8) sm.gate[(t - sg.a) * 8 + threadIdx.x] = __fmul_rn(sm.rows[threadIdx.x], nsc);
            cons_sync();
        }
        for (int t = su.a; t < su.b; t += su.per) {
            const int k = min(su.per, su.b - t);
            if (!unit_rows(dm, L.up, k, sm, rg)) return false;
            if (threadIdx.x < k * 8)
                swiglu(t * 8 + threadIdx.x, sm.gate[(t - su.a) * 8 + threadIdx.x],
                       __fmul_rn(sm.rows[threadIdx.x], nsc));
            cons_sync();
        }
    }
    tk.tr.stamp(ev, 2);
    return true;
}

// K5: x += Wdown act (cpu.go:347-350).
// The down product on a half tile: rows r0..r0+3 of tile t, two warps per row
// (each half of the blocks), the residual add in the epilogue.
__device__ bool ph_down_half(const DecParams &dm, int l, const Tok &tk, const DecSmem &sm, Ring &rg, int hh) {
    const Layer &L = lay(sm, tk, l);
    const QMat &m = L.down;
    const int t = hh >> 1, r0 = (hh & 1) * 4, row0 = t * 8 + r0;
    const uint32_t tact = tag_of(tk.epoch, dm.layers, l, PH_GU), tin = tag_of(tk.epoch, dm.layers, l, PH_O);
    const int ev = l * 5 + PH_DOWN;
    tk.tr.stamp(ev, 0);
    if (cons_or(!poll_stage_res(dm.ll_act, dm.ff, tact, sm.xv, m.type == 8 ? sm.xq8 : nullptr, dm.ll_x + row0, 4,
                                tin, sm.gate, dm.err) ||
                !slot_wait(sm.full, rg.sl, rg.ph, dm.err)))
        return false;
    tk.tr.stamp(ev, 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint8_t *slot = sm.ring + (size_t)rg.sl * rg.slot_bytes;
    const int hb = m.nb >> 1, b0 = (warp & 1) * hb, b1 = (warp & 1) ? m.nb : hb;
    const float a = dot_row(m.type, slot, m.nb, r0 + (warp >> 1), sm, lane, b0, b1);
    float *part = reinterpret_cast<float *>(sm.part);
    if (lane == 0) part[warp] = a;
    cons_sync();  // the slot is read: the feeder may refill it
    rg.next();
    if (threadIdx.x == kFeeder) feed_issue(sm, rg.nslots, rg.slot_bytes);
    if (threadIdx.x < 4) {
        const float v = __fadd_rn(part[2 * threadIdx.x], part[2 * threadIdx.x + 1]);
        ll_put(dm.ll_x + row0 + threadIdx.x, __fadd_rn(sm.gate[threadIdx.x], v),
               tag_of(tk.epoch, dm.layers, l, PH_DOWN));
    }
    tk.tr.stamp(ev, 2);
    return true;
}

__device__ bool ph_down(const DecParams &dm, int l, const Tok &tk, const DecSmem &sm, Ring &rg) {
    const Layer &L = lay(sm, tk, l);
    const Share s = share_of(sm, SK_DOWN, L.down);
    if (s.b <= s.a) return true;
    if (sm.st->down_half) return ph_down_half(dm, l, tk, sm, rg, s.a);
    const int F = dm.ff;
    const uint32_t tact = tag_of(tk.epoch, dm.layers, l, PH_GU), tin = tag_of(tk.epoch, dm.layers, l, PH_O);
    const int ev = l * 5 + PH_DOWN;
    tk.tr.stamp(ev, 0);
    if (cons_or(!poll_stage_res(dm.ll_act, F, tact, sm.xv, L.down.type == 8 ? sm.xq8 : nullptr, dm.ll_x + s.a * 8,
                                (s.b - s.a) * 8, tin, sm.gate, dm.err) ||
                !slot_wait(sm.full, rg.sl, rg.ph, dm.err)))
        return false;
    tk.tr.stamp(ev, 1);
    const uint32_t tag = tag_of(tk.epoch, dm.layers, l, PH_DOWN);
    for (int t = s.a; t < s.b; t += s.per) {
        const int k = min(s.per, s.b - t);
        if (!unit_rows(dm, L.down, k, sm, rg, t == s.a)) return false;
        if (threadIdx.x < k * 8) {
            const int row = t * 8 + threadIdx.x;
            ll_put(dm.ll_x + row, __fadd_rn(sm.gate[row - s.a * 8], sm.rows[threadIdx.x]), tag);
        }
        cons_sync();
    }
    tk.tr.stamp(ev, 2);
    return true;
}

// The head: RMSNorm(output_norm), logits, this CTA's argmax partial.
// One unit of the head (k tiles from tile t0): logits = (W h) * nsc
// (cpu.go:357-363), stored, and folded into this thread's running argmax.
// With more than 4 tiles each warp takes whole tiles and the lanes holding a
// row's value finish it, so a unit costs the slot's wait and its release;
// with fewer, a tile's blocks are split across warps and meet in shared
// memory first.
__device__ __forceinline__ bool head_unit(const DecParams &dm, int k, int t0, float nsc, const DecSmem &sm, Ring &rg,
                                          float &bv, int &bi) {
    const QMat &m = dm.head;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sl = rg.sl;
    bool ok = true;
    if (!mbar_try_wait(sm.full + sl, rg.ph)) {
        const uint64_t t0w = gtimer();
        while (!mbar_try_wait(sm.full + sl, rg.ph)) {
            if (read_err(dm.err)) {
                ok = false;
                break;
            }
            if (gtimer() - t0w > kWaitNs) {
                atomicExch(dm.err, DEV_RING_TIMEOUT);
                ok = false;
                break;
            }
        }
    }
    if (cons_or(!ok)) return false;
    const uint8_t *slot = sm.ring + (size_t)sl * rg.slot_bytes;
    auto finish = [&](int tile, int r, float a) {
        const int row = (t0 + tile) * 8 + r;
        const float v = __fmul_rn(a, nsc);
        if (row < dm.vocab) {
            dm.logits[row] = v;
            if (better(v, row, bv, bi)) bv = v, bi = row;
        }
    };
    if (2 * k > kCons) {
        for (int i = warp; i < k; i += kCons) {
            float a = dot_tile(m.type, slot + (size_t)i * m.tile_bytes, m.nb, sm, 0, m.nb, lane);
            a += __shfl_xor_sync(kFull, a, 1);
            a += __shfl_xor_sync(kFull, a, 2);
            if ((lane & 3) == 0) finish(i, lane >> 2, a);
        }
    } else {
        const int lg = k == 2 ? 2 : k <= 4 ? 1 : 0;  // parts = kCons / k = 1 << lg (k in 2..7), by shifts
        const int parts = 1 << lg;
        const int tile = warp >> lg, part = warp & (parts - 1);
        float a = 0.f;
        if (tile < k) {
            const int b0 = (m.nb * part) >> lg, b1 = (m.nb * (part + 1)) >> lg;
            a = dot_tile(m.type, slot + (size_t)tile * m.tile_bytes, m.nb, sm, b0, b1, lane);
        }
        a += __shfl_xor_sync(kFull, a, 1);
        a += __shfl_xor_sync(kFull, a, 2);
        float *part_s = reinterpret_cast<float *>(sm.part);
        if ((lane & 3) == 0) part_s[(lane >> 2) * 8 + warp] = a;
        cons_sync();
        if (threadIdx.x < 64) {
            float v = part_s[threadIdx.x];
            const int w = threadIdx.x & 7;
            if (parts >= 2) v += __shfl_xor_sync(kFull, v, 1);
            if (parts >= 4) v += __shfl_xor_sync(kFull, v, 2);
            if (parts >= 8) v += __shfl_xor_sync(kFull, v, 4);
            if ((w & (parts - 1)) == 0 && (w >> lg) < k) finish(w >> lg, threadIdx.x >> 3, v);
        }
    }
    cons_sync();  // the slot (and the shared partials) are free
    rg.next();
    if (threadIdx.x == kFeeder) feed_issue(sm, rg.nslots, rg.slot_bytes);
    return true;
}

__device__ bool ph_head(const DecParams &dm, const Tok &tk, const DecSmem &sm, Ring &rg) {
    const Share s = share_of(sm, SK_HEAD, dm.head);
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    const int ev = dm.layers * 5;
    tk.tr.stamp(ev, 0);
    if (s.b > s.a) {
        const int E = dm.embd;
        const uint32_t tin = tag_of(tk.epoch, dm.layers, dm.layers - 1, PH_DOWN);
        cp_async_wait_all();  // the norm weights, prefetched during the phase before
        cons_sync();
        const float ss = poll_stage(dm.ll_x, E, tin, sm.xv, dm.head.type == 8 ? sm.xq8 : nullptr, sm.nrm, dm.err);
        norm_partial(ss, sm);
        if (cons_or(ss < 0.f)) return false;
        tk.tr.stamp(ev, 1);
        const float nsc = norm_scale(dm, sm);
        for (int t = s.a; t < s.b; t += s.per)
            if (!head_unit(dm, min(s.per, s.b - t), t, nsc, sm, rg, bv, bi)) return false;
    }
    // CTA argmax over the threads that saw rows (all 8 warps reduce; idle lanes hold the identity)
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) sm.red[w] = bv, sm.red[kCons + w] = __int_as_float(bi);
    cons_sync();
    if (threadIdx.x == 0) {
        for (int k = 1; k < kCons; ++k) {
            const float v = sm.red[k];
            const int i = __float_as_int(sm.red[kCons + k]);
            if (better(v, i, bv, bi)) bv = v, bi = i;
        }
        // the token's argmax partial, released: every CTA's writes of the token
        // (its KV rows) are visible to a CTA that has read it and fenced
        __threadfence();
        uint64_t *dst = dm.ll_am + ((size_t)(tk.epoch & 1) * gridDim.x + blockIdx.x) * 2;
        const uint32_t tag = tag_of(tk.epoch, dm.layers, dm.layers - 1, PH_HEAD);
        ll_put(dst, bv, tag);
        ll_put(dst + 1, __int_as_float(bi), tag);
    }
    tk.tr.stamp(ev, 2);
    return true;
}

// The token: the argmax over every CTA's partial (polled, then fenced, so
// that the KV rows the CTAs wrote for this token are visible to this CTA's
// next reads); -1 on a device error.  Partials alternate between two buffers
// by token, and every CTA reads them all before its next token, so none is
// overwritten before it is read.
__device__ int argmax_partials(const DecParams &dm, const Tok &tk, const DecSmem &sm) {
    const uint32_t tag = tag_of(tk.epoch, dm.layers, dm.layers - 1, PH_HEAD);
    const Seg seg[1] = {{dm.ll_am + (size_t)(tk.epoch & 1) * gridDim.x * 2, 2 * (int)gridDim.x, tag, sm.xv}};
    const bool ok = poll_segs(seg, dm.err);
    __threadfence();
    if (cons_or(!ok)) return -1;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += kConsThreads) {
        const float v = sm.xv[2 * i];
        const int ix = __float_as_int(sm.xv[2 * i + 1]);
        if (better(v, ix, bv, bi)) bv = v, bi = ix;
    }
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) sm.red[w] = bv, sm.red[kCons + w] = __int_as_float(bi);
    cons_sync();
    if (threadIdx.x == 0) {
        for (int k = 1; k < kCons; ++k) {
            const float v = sm.red[k];
            const int i = __float_as_int(sm.red[kCons + k]);
            if (better(v, i, bv, bi)) bv = v, bi = i;
        }
        sm.red[2 * kCons] = __int_as_float(bi == 0x7fffffff ? 0 : bi);
    }
    cons_sync();
    return __float_as_int(sm.red[2 * kCons]);
}

// The token loop of the persistent kernel (returns early on a device error,
// which dm.err records).
__device__ __forceinline__ void decode_tokens(const DecParams &dm, int ntok, const DecSmem &sm,
                                              Ring &rg) {
    Tok tk;
    tk.pos = (int)__ldcg(dm.state), tk.step = (int)__ldcg(dm.state + 1);
    tk.tok = __ldcg(dm.tokens + tk.step);
    tk.epoch = __ldcg(dm.ll_epoch);
    fetch_layer(dm, sm, 0);
    fetch_layer(dm, sm, 1);
    for (int i = 0; i < ntok; ++i) {
        tk.g0 = i * dm.layers;
        if (tk.pos >= dm.ctx) {
            if (threadIdx.x == 0) atomicExch(dm.err, DEV_CONTEXT_FULL);
            return;
        }
        const int nch = (tk.pos + dm.dec_chunk) / dm.dec_chunk;
        tk.tr.p = (dm.trace && i == 0) ? dm.trace + (size_t)blockIdx.x * dm.trace_events * 4 : nullptr;
        if (threadIdx.x == 0) s_ring_wait = 0;
        if (blockIdx.x == 0) {  // the embedding row is the residual of layer 0
            for (int e = threadIdx.x; e < dm.embd; e += kConsThreads) {
                const QMat &m = dm.embed;
                const uint8_t *t = m.tiles + (size_t)(tk.tok >> 3) * m.tile_bytes;
                const int r = tk.tok & 7, b = e >> 5, j = e & 31, qb = m.type == 8 ? 32 : 16;
                const float d = __half2float(reinterpret_cast<const __half *>(t + (size_t)m.nb * 8 * qb)[b * 8 + r]);
                const uint8_t *qs = t + ((size_t)b * 8 + r) * qb;
                const float v = m.type == 8 ? d * (float)(int8_t)qs[j]
                                            : d * (float)(((j < 16) ? (qs[j & 15] & 15) : (qs[j & 15] >> 4)) - 8);
                ll_put(dm.ll_x + e, v, tag_of(tk.epoch, dm.layers, -1, PH_DOWN));
            }
        }
        cp_async_wait_all();  // layers 0 and 1 of the token
        cons_sync();
        qkv_prefetch(dm, 0, tk, sm);
        for (int l = 0; l < dm.layers; ++l) {
            if (l > 0) {  // layer l + 1's descriptor (and this layer's prefetches), then layer l + 2's copy
                cp_async_wait_all();
                cons_sync();
            }
            fetch_layer(dm, sm, tk.g0 + l + 2);
            if (!ph_qkv(dm, l, tk, sm, rg)) return;
            // attention items from the last CTA down: those have no QKV, output
            // or down rows, so they copy the K/V history well before q, k, v arrive
            for (int item = gridDim.x - 1 - blockIdx.x; item < dm.heads * nch; item += gridDim.x)
                if (!ph_attn(dm, l, tk, item, nch, sm)) return;
            if (sm.st->b[SK_GU] > sm.st->a[SK_GU]) prefetch_norm(lay(sm, tk, l).ffn_norm, dm.embd, sm);
            if (!ph_o(dm, l, tk, sm, rg)) return;
            if (!ph_gu(dm, l, tk, sm, rg)) return;
            if (l + 1 < dm.layers) qkv_prefetch(dm, l + 1, tk, sm);
            else prefetch_norm(dm.out_norm, dm.embd, sm);
            if (!ph_down(dm, l, tk, sm, rg)) return;
        }
        if (!ph_head(dm, tk, sm, rg)) return;
        tk.tr.stamp(dm.layers * 5 + 1, 0);
        const int tok = argmax_partials(dm, tk, sm);
        if (tok < 0) return;
        tk.tr.stamp(dm.layers * 5 + 1, 2);
        tk.tok = tok;
        tk.pos++, tk.step++, tk.epoch++;
        if (blockIdx.x == 0 && threadIdx.x == 0) dm.tokens[tk.step] = tk.tok;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        dm.state[0] = tk.pos;
        dm.state[1] = tk.step;
        *dm.ll_epoch = tk.epoch;
    }
}

__global__ void __launch_bounds__(kDecThreads, 1)
    k_decode2(const __grid_constant__ DecParams dm, int ntok, int nslots, int slot_bytes) {
    extern __shared__ __align__(128) uint8_t dsm[];
    DecSmem sm;
    {
        const DecLayout lo =
            dec_layout(nslots, slot_bytes, dm.embd, dm.ff, dm.head_dim, dm.heads, dm.dec_gate_rows, dm.dec_qkv_rows,
                       dm.feed_max, dm.dec_chunk);
        sm.ring = dsm + lo.ring;
        sm.full = reinterpret_cast<uint64_t *>(dsm + lo.full);
        sm.feed = reinterpret_cast<Feed *>(dsm + lo.feed);
        sm.plan = reinterpret_cast<FeedUnit *>(dsm + lo.plan);
        sm.lay = reinterpret_cast<Layer *>(dsm + lo.lay);
        sm.st = reinterpret_cast<ShareTab *>(dsm + lo.shares);
        sm.xv = reinterpret_cast<float *>(dsm + lo.xv);
        sm.xq8 = reinterpret_cast<float *>(dsm + lo.xq8);
        sm.xs = reinterpret_cast<float *>(dsm + lo.xs);
        sm.part = reinterpret_cast<double *>(dsm + lo.part);
        sm.rows = reinterpret_cast<float *>(dsm + lo.rows);
        sm.gate = reinterpret_cast<float *>(dsm + lo.gate);
        sm.red = reinterpret_cast<float *>(dsm + lo.red);
        sm.att = reinterpret_cast<float *>(dsm + lo.att);
        sm.merge = reinterpret_cast<float *>(dsm + lo.merge);
        sm.pre = reinterpret_cast<float *>(dsm + lo.pre);
        sm.kvs = reinterpret_cast<float *>(dsm + lo.kvs);
        sm.nrm = reinterpret_cast<float *>(dsm + lo.nrm);
    }
    if (threadIdx.x < 4 * SK_N) {  // the share table: a thread per entry
        const Layer &L0 = dm.layer[0];
        const int kind = threadIdx.x % SK_N, what = threadIdx.x / SK_N;
        const QMat &m = kind == SK_QKV ? L0.q : kind == SK_O ? L0.o : kind == SK_GU ? L0.gate
                                             : kind == SK_DOWN ? L0.down : dm.head;
        if (what == 0) {
            const bool half = kind == SK_DOWN && down_halves(m, gridDim.x);
            const int T = kind == SK_QKV ? (L0.q.rows + L0.k.rows + L0.v.rows) >> 3 : (m.rows >> 3) << (half ? 1 : 0);
            const int P = kind == SK_QKV ? dec_qkv_ctas(T, gridDim.x, dm.heads) : min((int)gridDim.x, T);
            const int cta = blockIdx.x;
            sm.st->a[kind] = cta < P ? split_at(T, cta, P) : 0;
            sm.st->b[kind] = cta < P ? split_at(T, cta + 1, P) : 0;
            if (kind == SK_DOWN) sm.st->down_half = half;
        } else {
            const int type = what == 1 ? 2 : what == 2 ? 3 : 8;  // formats in fmt_ix order
            sm.st->per[kind][what - 1] = max(1, min(kConsThreads / 8, slot_bytes / tile_bytes_of(type, m.nb)));
        }
    }
    const int nplan = __ldg(dm.feed_count + blockIdx.x);
    for (int j = threadIdx.x; j < nplan; j += kConsThreads)
        sm.plan[j] = dm.feed_plan[(size_t)blockIdx.x * kMaxFeedPlan + j];
    if (threadIdx.x == 0) {
        s_wait_ns = dm.wait_ns ? dm.wait_ns : kWaitNs;
        for (int i = 0; i < nslots; ++i) mbar_init(sm.full + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *sm.feed = Feed{0, 0, 0, 0, 0u, 0, nplan, (unsigned)(ntok * nplan), 0};
    }
    __syncthreads();
    if (threadIdx.x == kFeeder)
        for (int i = 0; i < nslots; ++i) feed_issue(sm, nslots, slot_bytes);
    Ring rg{nslots, slot_bytes, 0u, 0, 0u};
    decode_tokens(dm, ntok, sm, rg);
    cp_async_wait_all();  // descriptor copies of layers past the launch's last
    if (threadIdx.x == kFeeder) feed_drain(sm, nslots, rg.u);
}

}  // namespace

DecConfig decode_config(const Shapes &s, int max_tile_bytes, int head_tile_bytes, int gate_rows, int qkv_rows,
                        int plan_units, int attn_positions) {
    // A ring of 4 slots of at least 16 KB runs far enough ahead of the
    // consumers; the attention item's K/V rows take what is left.
    DecConfig c{};
    const int budget = 232448 - 1024;  // the opt-in maximum per block, less the static shared memory
    auto total = [&](int nslots, int slot, int chunk) {
        return dec_layout(nslots, slot, s.embd, s.ff, s.head_dim, s.heads, gate_rows, qkv_rows, plan_units, chunk).total;
    };
    // The slot size is chosen before the weight plan is listed (the plan depends on it) and again after, with
    // room for at least 512 plan units both times, so that both choices agree.
    const int ring = budget - (int)dec_layout(0, 0, s.embd, s.ff, s.head_dim, s.heads, gate_rows, qkv_rows,
                                              max(plan_units, 512), 64).total;
    int slot = max(max_tile_bytes, 16384);
    // The head streams back to back and each unit costs two consumer barriers and a slot wait: a slot of
    // 8 head tiles (when small) gives each warp a tile per unit; larger heads take as many tiles per unit
    // (4, else 2) as 4 slots leave room for.
    if (8 * head_tile_bytes <= 24576) {
        slot = max(slot, 8 * head_tile_bytes);
    } else {
        for (int mult = 4; mult >= 2; mult >>= 1) {
            const int s2 = (max(slot, mult * head_tile_bytes) + 127) / 128 * 128;
            if (4 * s2 <= ring) {
                slot = s2;
                break;
            }
        }
    }
    slot = (slot + 127) / 128 * 128;
    c.slot_bytes = slot;
    c.nslots = min(4, ring / slot);
    // Positions per attention item: a head's whole context in one item when
    // it fits saves the exchange of partials between CTAs, which outweighs
    // the L1 a full block of shared memory takes (measured: 224 positions ran
    // 2.5 % faster than 192 on the SmolLM2 shape, whose contexts reach 256).
    // By default the most that fit, a multiple of 32 up to 256 (a lane per
    // position of a warp's share).
    c.chunk = 64;
    for (int k = attn_positions > 0 ? attn_positions : 256; k > 64; k -= 32)
        if (total(c.nslots, slot, k) <= (size_t)budget) {
            c.chunk = k;
            break;
        }
    c.smem = total(c.nslots, slot, c.chunk);
    c.threads = kDecThreads;
    return c;
}

cudaError_t launch_decode2(const DecParams &dm, const DecConfig &c, int ntok, int ctas,
                           cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(k_decode2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(c.threads);
    cfg.dynamicSmemBytes = c.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_decode2, dm, ntok, c.nslots, c.slot_bytes);
}

cudaError_t launch_feed_plan(const DecParams &dm, int slot_bytes, FeedUnit *plan, int *count, int ctas,
                             cudaStream_t st) {
    k_feed_plan<<<ctas, 32, 0, st>>>(dm, slot_bytes, plan, count);
    return cudaGetLastError();
}

int decode2_ctas_per_sm(const DecConfig &c) {
    int n = 0;
    cudaFuncSetAttribute(k_decode2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_decode2, c.threads, c.smem);
    return n;
}

}  // namespace llmb
