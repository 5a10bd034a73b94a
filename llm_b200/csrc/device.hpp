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
constexpr int kSsqTiles = 8;       // 128-row tiles of a residual row (embd <= 1024)

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

struct alignas(16) Layer {  // 16-byte aligned: the decode kernel copies it in 16-byte pieces
    QMat q, k, v;  // q and k rows in adjacent-pair RoPE order (NEOX rows permuted at load)
    QMat o, gate, up, down;
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
    const float *bq = nullptr, *bk = nullptr, *bv = nullptr;  // qwen2 biases (q, k permuted like their rows)
    float *kv = nullptr;  // [2][ctx][kvd]: K at 0, V at ctx * kvd (fused.go:221, kernels_fused.go:440-445)
};

// What the kernels need besides the per-layer descriptors.
// A batch of up to kMaxPrefill tokens from any sequences (multi-stream
// decode, and prompt tokens of several sequences): token t (residual row t
// of x) sits at position pos[t] of the sequence whose KV cache is slot[t] of
// the arena (slot s, layer l at kv + (s * layers + l) * 2 * ctx * kvd, K
// then V as in Layer::kv).  The batch head writes the argmax of row
// head_rows[j] to out[j].
struct TokBatch {
    int pos[kMaxPrefill];
    int slot[kMaxPrefill];
    int tok[kMaxPrefill];
    int head_rows[kMaxPrefill];
    int out[kMaxPrefill];
    float *kv;
    int layers;
};

// One unit of a CTA's weight stream in the persistent decode kernel: one or
// two source ranges copied into one ring slot.
struct FeedUnit {
    const uint8_t *src1, *src2;
    uint32_t n1, n2;
};
constexpr int kMaxFeedPlan = 1024;  // units of one token per CTA

struct ModelHeader {
    int embd, ff, heads, kv_heads, head_dim, kvd, vocab, ctx, layers;
    float eps, scale;  // RMSNorm epsilon; 1/sqrt(head_dim) (cpu.go:304)
    int rope_neox;
    QMat embed, head;  // token_embd (the gather) and the output matrix (token_embd when tied)
    const float *out_norm;
    const float *rope_cs;  // [ctx][head_dim/2][2] cos, sin (gpu.go:524-534)

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
    // the m-token products (gemm.cu): normed rows [kMaxPrefill][embd], the
    // head's per (token, row tile) argmax partials
    float *h;
    float2 *gam;
    // the tensor-core products' RMSNorm inputs: per token, the sums of squares of the residual row over
    // each 128-row tile ([kMaxPrefill][kSsqTiles], written by the embedding and the residual epilogues)
    float *ssq;

    // the persistent decode kernel's tagged activations ({f32 value, u32 tag})
    uint64_t *ll_x, *ll_q, *ll_k, *ll_v, *ll_att, *ll_act, *ll_pv, *ll_ml;
    uint64_t *ll_am;     // per token parity and CTA: the head's argmax partial {value, index}
    uint32_t *ll_epoch;  // tokens decoded so far by the persistent kernel (makes tags unique across calls)
    int dec_gate_rows;   // gate rows of the largest gate/up share of a CTA
    int dec_qkv_rows;    // rows of the largest QKV share of a CTA
    int dec_chunk;       // positions per attention item (a multiple of 32, 64..256)
    const Layer *layers_g;  // the layers' descriptors in device memory (the decode kernel stages them in shared memory)
    // each CTA's units of one token, in consumption order (plan[cta * kMaxFeedPlan + j],
    // feed_count[cta] of them; feed_max the largest count), built once per model
    const FeedUnit *feed_plan;
    const int *feed_count;
    int feed_max;
    // optional phase timeline of the persistent decode kernel (null: off):
    // trace[(cta * trace_events + event) * 4 + {0, 1, 2}] = globaltimer ns at
    // the phase's entry, when its input was ready, at its exit, and + 3 the
    // SM cycles it waited for weight slots; events are
    // 5 per layer (QKV, attention, output, gate/up, down), then head, then
    // the token's argmax exchange.  Recorded for the first token of a launch.
    uint64_t *trace;
    int trace_events;
    // the persistent decode kernel's limit on every wait (flag polls, weight
    // slots), in ns; 0 means the default of 2 s.  Past it the kernel records
    // DEV_TAG_TIMEOUT or DEV_RING_TIMEOUT in err and returns.
    uint64_t wait_ns;
    // a test aid for that error path: at the token whose step (state[1]) is
    // drop_step, CTA 0 does not publish its output-projection rows of layer
    // 0, so the gate/up phase's wait for them runs out.  -1: off.
    int drop_step;
};


// Everything a kernel needs (header + layers).  DevModel lives in device
// memory for the per-phase kernels; DecParams is the persistent decode
// kernel's __grid_constant__ parameter (constant memory, so the uniform
// descriptor reads of every phase hit the constant cache, not L1, which the
// kernel's large shared memory leaves small).
template <int NL>
struct ModelDesc : ModelHeader {
    Layer layer[NL];
};
constexpr int kMaxDecLayers = 64;
using DevModel = ModelDesc<kMaxLayers>;
using DecParams = ModelDesc<kMaxDecLayers>;
static_assert(sizeof(DecParams) < 32000, "kernel parameters are limited to 32 KB");

// CTAs of the persistent decode kernel that take QKV rows (T tiles): the
// first ones, leaving the last `heads` CTAs, which take the attention items of
// a token's first context chunk, free to start their items (their K/V loads)
// while the QKV rows are computed.
__host__ __device__ inline int dec_qkv_ctas(int T, int ncta, int heads) {
    const int p = ncta - heads > ncta / 2 ? ncta - heads : ncta;
    return T < p ? T : p;
}

// Shared-memory layout of the persistent decode kernel (byte offsets).
struct DecLayout {
    size_t ring, full, feed, plan, lay, shares, xv, xq8, xs, part, rows, gate, red, att, merge, pre, kvs, nrm, total;
};

__host__ __device__ inline DecLayout dec_layout(int nslots, int slot_bytes, int embd, int ff, int head_dim, int heads,
                                                int gate_rows, int qkv_rows, int plan_units, int dec_chunk) {
    DecLayout l{};
    const size_t vec = (size_t)((embd > ff ? embd : ff) + 31) / 32 * 36 * 4;  // 32-wide blocks padded to 36 floats
    size_t p = 0;
    l.ring = p, p += (size_t)nslots * slot_bytes;
    l.full = p, p += 8 * (size_t)nslots;
    l.feed = p, p += 64;
    l.plan = p, p += sizeof(FeedUnit) * (size_t)plan_units;
    p = (p + 15) / 16 * 16;
    l.lay = p, p += 3 * sizeof(Layer);
    l.shares = p, p += 128;  // ShareTab (decode.cu)
    p = (p + 127) / 128 * 128;
    l.xv = p, p += vec;
    l.xq8 = p, p += vec;
    l.xs = p, p += vec;
    l.part = p, p += 8 * 64;
    l.rows = p, p += 4 * 256;
    l.gate = p, p += 4 * (size_t)gate_rows;
    // an attention item's history K rows [dec_chunk][head_dim + 4] and V rows
    // [dec_chunk][head_dim] share the bytes of the matrix phases' vectors
    // above (no phase uses both); with head_dim 64 the item keeps them in
    // registers
    l.kvs = l.xv;
    const size_t kv_end = l.kvs + (head_dim == 64 ? 0 : 4 * (size_t)dec_chunk * (2 * head_dim + 4));
    p = p > kv_end ? p : kv_end;
    p = (p + 15) / 16 * 16;
    l.red = p, p += 4 * 64;
    l.att = p, p += 4 * (size_t)(3 * head_dim + 8 * (head_dim + 4));
    p = (p + 15) / 16 * 16;
    l.merge = p, p += 4 * (size_t)(9 * head_dim + 32);
    p = (p + 15) / 16 * 16;
    l.pre = p, p += 4 * (size_t)(4 * qkv_rows);
    p = (p + 15) / 16 * 16;
    l.nrm = p, p += 4 * (size_t)embd;
    l.total = (p + 127) / 128 * 128;
    return l;
}

}  // namespace llmb
