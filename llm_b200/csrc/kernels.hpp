// Host-side launchers of the forward-pass kernels (kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include "device.hpp"

namespace llmb {

// Device error codes written to DevModel::err.
enum DeviceError : int {
    DEV_OK = 0,
    DEV_BARRIER_TIMEOUT = 1,  // reserved: a grid-wide barrier waited longer than its limit (none is used now)
    DEV_CONTEXT_FULL = 2,     // a token past the context
    DEV_TAG_TIMEOUT = 3,      // a tagged activation did not arrive in time
    DEV_RING_TIMEOUT = 4,     // a weight slot did not fill or drain in time
    DEV_MMA_TIMEOUT = 5,      // the tensor cores did not signal a product's completion in time
};

// Host copy of what launch shapes need.
struct Shapes {
    int embd, ff, heads, kv_heads, head_dim, kvd, vocab, ctx, layers, nchunk;
    int qkv_tiles, o_tiles, gu_tiles, down_tiles, head_tiles;
    int head_ctas;  // CTAs of the head kernel (argmax partials)
};

constexpr int kWarps = 8;             // warps per CTA
constexpr int kThreads = kWarps * 32; // threads per CTA

// Dynamic shared memory of every kernel: a vector region, then reduction scratch.
int smem_vec_floats(const Shapes &s);
size_t smem_bytes(const Shapes &s);
// Lets the per-phase kernels use smem_bytes(s) of dynamic shared memory.
cudaError_t prepare_kernels(const Shapes &s);

// Repacks `rows` raw GGUF rows (blocks of `type`) staged in device memory
// into the tile layout at destination row dst_row0.  neox_hd > 0 reorders the
// rows of each head of neox_hd rows from the NEOX layout to adjacent pairs
// (fused.go:329-344): destination row nr takes source row neoxMap(nr).
void launch_repack(const uint8_t *raw, int rows, int nb, int type, uint8_t *tiles, int tile_bytes, int dst_row0,
                   int neox_hd, cudaStream_t st);

// The embedding rows of m tokens into x (the layer-0 kernels fold this in;
// used alone when no layer runs).
void launch_embed(const DevModel *dm, const Shapes &s, int m, cudaStream_t st, const TokBatch *tb = nullptr);

// One layer for m tokens at positions state.pos .. state.pos+m-1 of the
// model's sequence, or, with a TokBatch (device memory), token t at position
// tb->pos[t] of KV slot tb->slot[t] (5 kernels: norm+QKV+bias+RoPE+KV append,
// attention partials and merge, output projection + residual,
// norm+gate/up+SwiGLU, down + residual).
void launch_layer(const DevModel *dm, const Shapes &s, int l, int m, cudaStream_t st, const TokBatch *tb = nullptr);

// Final norm of token t_src's residual, the vocab logits, and the argmax:
// writes tokens[state.step + adv] and advances state by adv.
void launch_head(const DevModel *dm, const Shapes &s, int t_src, int adv, cudaStream_t st);

// The attention of one layer alone (the m-token path's products are in gemm.cu).
// pdl: launched as a programmatic dependent of the kernel before it (k_attn waits for it first)
cudaError_t launch_attention(const DevModel *dm, const Shapes &s, int l, int m, cudaStream_t st, const TokBatch *tb,
                             bool pdl = false);

// One layer for m <= 64 tokens through the chunked products of gemm.cu
// (norm, QKV product with bias/RoPE/KV append, attention, output product +
// residual, norm, gate/up product + SwiGLU, down product + residual); hd is
// the host copy of *dm (device pointers), nsm the SMs to fill.  tensor: the
// products on the tensor cores (k_mma, split bf16 pieces), else in float32 on
// the CUDA cores (k_gemm).
cudaError_t launch_layer_mm(const DevModel *dm, const DevModel &hd, const Shapes &s, int l, int m, int nsm,
                            cudaStream_t st, const TokBatch *tb, bool tensor);
// The head for `rows` residual rows listed at rows_dev (device): final norm,
// the vocabulary product and the argmax of each row into tb->out.
cudaError_t launch_head_mm(const DevModel *dm, const DevModel &hd, const Shapes &s, TokBatch *tb, const int *rows_dev,
                           int rows, int nsm, cudaStream_t st, bool tensor);
// Lets the tensor-core products use their dynamic shared memory (once per device).
cudaError_t prepare_products();

// The argmax of the residual rows tb->head_rows[0..rows) into tb->out.
void launch_head_batch(const DevModel *dm, const Shapes &s, TokBatch *tb, int rows, cudaStream_t st);

// state += n.
void launch_advance(const DevModel *dm, int n, cudaStream_t st);

// The warp-specialised persistent decode kernel (decode.cu).
struct DecConfig {
    int nslots, slot_bytes, threads, chunk;  // chunk: positions per attention item
    size_t smem;
};
DecConfig decode_config(const Shapes &s, int max_tile_bytes, int head_tile_bytes, int gate_rows, int qkv_rows,
                        int plan_units, int attn_positions);
// Each CTA's weight units of one token for the persistent kernel (its grid: ctas).
cudaError_t launch_feed_plan(const DecParams &dm, int slot_bytes, FeedUnit *plan, int *count, int ctas,
                             cudaStream_t st);
cudaError_t launch_decode2(const DecParams &dm, const DecConfig &c, int ntok, int ctas,
                           cudaStream_t st);
int decode2_ctas_per_sm(const DecConfig &c);

}  // namespace llmb
