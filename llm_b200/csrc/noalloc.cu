// Decode attention that allocates nothing: llmb_attention_noalloc.
//
// The same split-KV attention as the model's (per (head, chunk of 64
// positions) partials, then a merge; cpu.go:304-335 for the math), for
// callers that cannot allocate device memory.  Its scratch, the chunks'
// partials, is a file-scope __device__ array of a fixed size instead of a
// cudaMalloc'd buffer.  Every GPU that loads this library holds the array
// (about 1 MiB) until the process exits.
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <mutex>

#include "../../include/llm_b200.h"

namespace llmb {
namespace {

constexpr int kNaChunk = 64;                       // positions per partial
constexpr int kNaMaxHeads = 32;                    // query heads
constexpr int kNaMaxChunks = 64;                   // 4096 positions
constexpr int kNaMaxHeadDim = 128;
constexpr int kNaStride = kNaMaxHeadDim + 2;       // per (head, chunk): V sum, then max and sum of exp
constexpr int kNaThreads = 256;

// The scratch.  In host code this name is only a stand-in for the device
// array: the host passes the address cudaGetSymbolAddress returns.
static __device__ __align__(256) float g_scratch[kNaMaxHeads * kNaMaxChunks * kNaStride];

// Partial of (head h = blockIdx.y, chunk c = blockIdx.x): max score m, sum of
// exp l, exp-weighted V sum, accumulated in double.
__global__ void __launch_bounds__(kNaThreads) k_na_partial(const float *__restrict__ q, const float *__restrict__ kc,
                                                           const float *__restrict__ vc, int n, int heads,
                                                           int kv_heads, int hd, int stride, float scale,
                                                           float *scratch) {
    __shared__ float qs[kNaMaxHeadDim], e[kNaChunk], red[kNaThreads / 32];
    const int c = blockIdx.x, h = blockIdx.y, kvh = h / (heads / kv_heads);
    const int p0 = c * kNaChunk, cnt = min(kNaChunk, n - p0);
    for (int i = threadIdx.x; i < hd; i += kNaThreads) qs[i] = q[h * hd + i];
    __syncthreads();
    // scores: 4 threads per position
    const int p = threadIdx.x >> 2, sub = threadIdx.x & 3;
    double ps = 0.0;
    if (p < cnt)
        for (int d = sub; d < hd; d += 4) ps = fma((double)qs[d], (double)kc[(size_t)(p0 + p) * stride + kvh * hd + d], ps);
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    const float s = p < cnt ? __fmul_rn((float)ps, scale) : -FLT_MAX;
    float m = s;
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < kNaThreads / 32; ++w) m = fmaxf(m, red[w]);
    if (p < cnt && sub == 0) e[p] = (float)exp((double)__fsub_rn(s, m));
    __syncthreads();
    float *out = scratch + ((size_t)h * kNaMaxChunks + c) * kNaStride;
    // V sum: thread d of the head over the chunk's positions
    for (int d = threadIdx.x; d < hd; d += kNaThreads) {
        double o = 0.0;
        for (int pp = 0; pp < cnt; ++pp) o = fma((double)e[pp], (double)vc[(size_t)(p0 + pp) * stride + kvh * hd + d], o);
        out[d] = (float)o;
    }
    if (threadIdx.x == 0) {
        double l = 0.0;
        for (int pp = 0; pp < cnt; ++pp) l += e[pp];
        out[kNaMaxHeadDim] = m;
        out[kNaMaxHeadDim + 1] = (float)l;
    }
}

// Merge of head h's chunks: sum_c e^{m_c-M} pv_c / sum_c e^{m_c-M} l_c.
__global__ void __launch_bounds__(kNaThreads) k_na_merge(int n, int hd, const float *scratch, float *att) {
    const int h = blockIdx.x, nch = (n + kNaChunk - 1) / kNaChunk;
    const float *base = scratch + (size_t)h * kNaMaxChunks * kNaStride;
    for (int d = threadIdx.x; d < hd; d += kNaThreads) {
        double M = -1e300;
        for (int c = 0; c < nch; ++c) M = fmax(M, (double)base[c * kNaStride + kNaMaxHeadDim]);
        double l = 0.0, o = 0.0;
        for (int c = 0; c < nch; ++c) {
            const double f = exp((double)base[c * kNaStride + kNaMaxHeadDim] - M);
            l = fma(f, (double)base[c * kNaStride + kNaMaxHeadDim + 1], l);
            o = fma(f, (double)base[c * kNaStride + d], o);
        }
        att[(size_t)h * hd + d] = (float)(o / l);
    }
}

// The scratch's device address per device.  Outside stream capture every
// call looks it up again with that device current (cudaGetSymbolAddress is a
// host-side query; it allocates nothing), so an address never outlives the
// context it belongs to (a cudaDeviceReset, or another context made current
// on the device, gets a fresh one).  A call made while its stream captures a
// graph uses the address its device's last call outside capture found.
std::mutex g_mu;
float *g_addr[64];

}  // namespace
}  // namespace llmb

using namespace llmb;

extern "C" LLMB_API int llmb_attention_noalloc(const float *q, const float *k_cache, const float *v_cache, int n_pos,
                                               int heads, int kv_heads, int head_dim, int kv_stride, float *out,
                                               void *stream) {
    if (!q || !k_cache || !v_cache || !out || n_pos <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 ||
        head_dim <= 0 || kv_stride < kv_heads * head_dim)
        return LLMB_ERR_ARG;
    if (heads > kNaMaxHeads || head_dim > kNaMaxHeadDim || n_pos > kNaMaxChunks * kNaChunk)
        return LLMB_ERR_ARG;  // beyond the fixed scratch: at most 32 heads, head_dim 128, 4096 positions
    // An error left pending by earlier work is the caller's: report it without
    // clearing it and without launching.
    if (cudaPeekAtLastError() != cudaSuccess) return LLMB_ERR_CUDA;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LLMB_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return LLMB_ERR_CUDA;
    float *scratch;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (cap == cudaStreamCaptureStatusNone) {
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || !p) return LLMB_ERR_CUDA;
            g_addr[dev] = static_cast<float *>(p);
        } else if (!g_addr[dev]) {
            return LLMB_ERR_CUDA;  // the first call on a device must come before any capture
        }
        scratch = g_addr[dev];
    }
    const int nch = (n_pos + kNaChunk - 1) / kNaChunk;
    const float scale = (float)(1.0 / std::sqrt((double)head_dim));  // cpu.go:304
    k_na_partial<<<dim3(nch, heads), kNaThreads, 0, st>>>(q, k_cache, v_cache, n_pos, heads, kv_heads, head_dim,
                                                          kv_stride, scale, scratch);
    if (cudaGetLastError() != cudaSuccess) return LLMB_ERR_CUDA;  // this launch's own error (none was pending)
    k_na_merge<<<heads, kNaThreads, 0, st>>>(n_pos, head_dim, scratch, out);
    return cudaGetLastError() == cudaSuccess ? LLMB_OK : LLMB_ERR_CUDA;
}
