// Device-side model description shared by the host code and the kernels.
//
// Weight layout in HBM.  The reference splits each GGUF block into a quant
// array and an f32 scale array (gpu.go:287-391).  Here a quantised matrix is
// cut into tiles of 8 consecutive output rows; a tile holds, for each 32-wide
// block b of the row, the 8 rows' quant bytes side by side, then the 8 rows'
// binary16 scales (and, for Q4_1, their binary16 minima):
//
//   tile = qs[nb][8][QB] | d[nb][8] (f16) | m[nb][8] (f16, Q4_1 only)
//   QB = 16 bytes (Q4_0, Q4_1) or 32 bytes (Q8_0)
//
// so a warp (8 rows x 4 lanes) reads one block of all 8 rows as 128 or 256
// contiguous bytes, and a CTA's share of a matrix is one contiguous range.
// Scales stay in binary16 (converted exactly in registers), so the bytes a
// kernel reads equal the GGUF bytes: 18 per 32 weights for Q4_0, 20 for
// Q4_1, 34 for Q8_0.  Rows are padded to a multiple of 8 with zero rows.
#pragma once

#include <cstdint>

namespace llmb {

constexpr int kTileRows = 8;
constexpr int kMaxLayers = 256;
constexpr int kAttnChunk = 64;     // positions per attention partial (flash-decoding split)
constexpr int kMaxPrefill = 64;    // tokens per prefill chunk (PrefillBatch, gpu.go:165)
constexpr int kMaxDecodeBatch = 16; // MaxBatch, gpu.go:1046

struct QMat {
    const uint8_t *tiles = nullptr;  // tile t at tiles + t * tile_bytes
    int type = 0;                    // GGML_Q4_0, GGML_Q4_1 or GGML_Q8_0
    int nb = 0;                      // 32-wide blocks per row
    int rows = 0;                    // rows, a multiple of 8 (zero rows pad the last tile)
    int tile_bytes = 0;
};

__host__ __device__ inline int quant_bytes(int type) { return type == 8 ? 32 : 16; }

__host__ __device__ inline int tile_bytes_of(int type, int nb) {
    int per_block = kTileRows * (quant_bytes(type) + 2 + (type == 3 ? 2 : 0));
    return per_block * nb;
}

struct Layer {
    QMat q, k, v;  // q and k rows in adjacent-pair RoPE order (NEOX rows permuted at load)
    QMat o, gate, up, down;
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
    const float *bq = nullptr, *bk = nullptr, *bv = nullptr;  // qwen2 biases (q, k permuted like their rows)
    float *kv = nullptr;  // [2][ctx][kvd]: K at 0, V at ctx * kvd (fused.go:221, kernels_fused.go:440-445)
};

// Everything a kernel needs, resident in device memory (one per model).
struct DevModel {
    int embd, ff, heads, kv_heads, head_dim, kvd, vocab, ctx, layers;
    float eps, scale;  // RMSNorm epsilon; 1/sqrt(head_dim) (cpu.go:304)
    int rope_neox;
    QMat embed, head;  // token_embd (the gather) and the output matrix (token_embd when tied)
    const float *out_norm;
    const float *rope_cs;  // [ctx][head_dim/2][2] cos, sin (gpu.go:524-534)
    Layer layer[kMaxLayers];

    // activations
    float *x;       // residual stream [kMaxPrefill][embd]
    float *q;       // [kMaxPrefill][heads * head_dim]
    float *att;     // merged attention [kMaxPrefill][heads * head_dim] (Peek "att")
    float *act;     // SwiGLU output [kMaxPrefill][ff]
    float *logits;  // [vocab]
    float *part_pv; // attention partials [kMaxPrefill][heads][nchunk][head_dim]
    float2 *part_ml;// [kMaxPrefill][heads][nchunk] (max, sum of exp)
    int nchunk;     // ceil(ctx / kAttnChunk)
    uint32_t *att_cnt;  // [kMaxPrefill][heads] chunks of a head finished (the last one merges)
    int smem_vec;   // floats of the shared vector region; the reduction scratch follows
    // sampling
    uint32_t *state;   // {position, step} (gpu.go:840, kernels.go:397-415)
    int32_t *tokens;   // [ctx + 1] prompt, then the sampled tokens
    float2 *am_part;   // argmax partials per CTA (value, index as float bits)
    uint32_t *am_count;// arrival counter of the head kernel's CTAs
    int *err;          // device error word (0 = none)
};

}  // namespace llmb
