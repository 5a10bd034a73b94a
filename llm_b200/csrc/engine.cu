// The host side of the forward pass and the C ABI (include/llm_b200.h).
//
// Restates the reference's llm.GPU (gpu.go:116-1054, fused.go:72-320) over
// CUDA: NewGPU's loader, the prefill chunks, the decode loop with on-device
// sampling and token feedback, PrefillLogits and Peek.  The WebGPU plumbing
// (bind groups, buffer-size limits, submit budgets) has no counterpart; the
// kernels are in kernels.cu.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <map>
#include <vector>

#include "../../include/llm_b200.h"
#include "device.hpp"
#include "gguf.hpp"
#include "kernels.hpp"

namespace llmb {
namespace {

// Knobs: the reference's package variables (gpu.go:165,1052; Limits.MemoryBudget gpu.go:35).
std::atomic<int64_t> g_decode_batch{8};
std::atomic<int64_t> g_prefill_batch{kMaxPrefill};
std::atomic<int64_t> g_memory_budget{0};
std::atomic<int64_t> g_decode_mode{0};  // 0: persistent kernel, 1: per-phase kernels
std::atomic<int64_t> g_decode_trace{0};  // 1: record the persistent kernel's phase timeline (llmb_peek "trace")
std::atomic<int64_t> g_prefill_mode{0};   // 0: chunked products on the tensor cores, 1: the per-token kernels,
                                          // 2: chunked products in float32 on the CUDA cores (gemm.cu)
std::atomic<int64_t> g_tag_reset{0};      // > 0: reset the decode kernel's tags after that many tokens (a test aid)
std::atomic<int64_t> g_attn_positions{0}; // positions per attention item of the decode kernel (0: as many as fit)
std::atomic<int64_t> g_wait_limit_us{0};  // the decode kernel's limit on each wait, microseconds (0: 2 s)
std::atomic<int64_t> g_drop_publish{-1};  // a test aid: the step at which the decode kernel skips one publish

thread_local std::string t_open_error;

constexpr uint64_t kPieceSize = 4ull << 20;  // PieceSize, gpu.go:23

struct Error {
    int code;
    std::string msg;
};

double now_ms() {
    using namespace std::chrono;
    return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

}  // namespace

struct Model {
    int device = 0;
    Config cfg;
    Shapes sh{};
    DevModel hdm{};  // host copy of the device description
    DevModel *dm = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev2 = nullptr, ev3 = nullptr;
    cudaEvent_t lev[4][3] = {};  // per decode launch: start, end, tokens copied
    int lk[2] = {0, 0};          // lev index of each launch in flight
    std::vector<void *> allocs;
    std::vector<size_t> sizes;
    uint64_t used = 0, budget = 0;
    int pm = kMaxPrefill;  // tokens per prefill chunk
    int layers_run = 0;    // GPU.Layers (0: all)
    int persistent_ctas = 0;
    DecConfig dec{};
    std::unique_ptr<DecParams> dp;  // the decode kernel's parameter block (header + layers)
    int32_t *h_tokens = nullptr;  // pinned: prompt upload and sampled-token read-back
    TokBatch *tb = nullptr;       // multi-stream: the token batch (device) and its pinned staging copy
    TokBatch *h_tb = nullptr;
    float *bkv = nullptr;         // multi-stream: the KV arena, bkv_slots sequences
    int bkv_slots = 0;
    int64_t ll_tokens = 0;        // tokens the persistent kernel decoded since its tags were last reset
    // the m-token layer sequences (embedding + every layer's launches), captured once per
    // (tokens, batch or single sequence, layers) and replayed: a step of 64 sequences is ~210 launches
    std::map<int64_t, cudaGraphExec_t> graphs;
    uint32_t *h_state = nullptr;
    int *h_err = nullptr;
    llmb_stats stats{};
    std::string last_error;

    ~Model() {
        if (st) cudaStreamSynchronize(st);
        for (void *p : allocs) cudaFree(p);
        if (h_tokens) cudaFreeHost(h_tokens);
        if (h_tb) cudaFreeHost(h_tb);
        for (auto &g : graphs) cudaGraphExecDestroy(g.second);
        if (h_state) cudaFreeHost(h_state);
        if (h_err) cudaFreeHost(h_err);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        if (ev2) cudaEventDestroy(ev2);
        if (ev3) cudaEventDestroy(ev3);
        for (auto &l : lev)
            for (auto &e : l)
                if (e) cudaEventDestroy(e);
        if (st) cudaStreamDestroy(st);
    }

    // gpu.go:170-185: a device buffer, checked against the memory budget.
    template <class T>
    T *alloc(size_t bytes, Error &err) {
        bytes = (bytes + 255) / 256 * 256;
        if (used + bytes > budget) {
            err = {LLMB_ERR_MEMORY, "llm: the model needs more GPU memory than the " + std::to_string(budget) +
                                        " bytes granted"};
            return nullptr;
        }
        void *p = nullptr;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) {
            err = {LLMB_ERR_MEMORY, std::string("llm: cudaMalloc: ") + cudaGetErrorString(e)};
            return nullptr;
        }
        cudaMemsetAsync(p, 0, bytes, st);
        allocs.push_back(p);
        sizes.push_back(bytes);
        used += bytes;
        return static_cast<T *>(p);
    }

    void release(void *p) {
        for (size_t i = 0; i < allocs.size(); i++)
            if (allocs[i] == p) {
                cudaStreamSynchronize(st);
                cudaFree(p);
                used -= sizes[i];
                allocs.erase(allocs.begin() + i);
                sizes.erase(sizes.begin() + i);
                return;
            }
    }
};

namespace {

#define CUDA_TRY(expr)                                                                  \
    do {                                                                                \
        cudaError_t _e = (expr);                                                        \
        if (_e != cudaSuccess) return Error{LLMB_ERR_CUDA, std::string(#expr ": ") + cudaGetErrorString(_e)}; \
    } while (0)

// ------------------------------------------------------------- loading --

struct Loader {
    Model &m;
    const GgufFile &f;
    const ReadAt &read;
    uint8_t *pinned[2] = {nullptr, nullptr};
    uint8_t *staging[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int k = 0;

    ~Loader() {
        if (m.st) cudaStreamSynchronize(m.st);  // the last repack kernels still read staging
        for (int i = 0; i < 2; i++) {
            if (done[i]) cudaEventSynchronize(done[i]), cudaEventDestroy(done[i]);
            if (pinned[i]) cudaFreeHost(pinned[i]);
            if (staging[i]) cudaFree(staging[i]);
        }
    }

    Error init() {
        for (int i = 0; i < 2; i++) {
            CUDA_TRY(cudaHostAlloc(&pinned[i], kPieceSize, cudaHostAllocDefault));
            CUDA_TRY(cudaMalloc(&staging[i], kPieceSize));
            CUDA_TRY(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
        }
        return {LLMB_OK, ""};
    }

    // Reads [off, off+len) of the file into the next pinned buffer and copies
    // it to device staging; returns the staging buffer (stream-ordered).
    Error piece(uint64_t off, uint64_t len, uint8_t **dev) {
        const int i = k++ & 1;
        CUDA_TRY(cudaEventSynchronize(done[i]));  // the copy out of this buffer two pieces ago
        if (read(off, pinned[i], len) < len) return {LLMB_ERR_IO, "llm: short read of the model file"};
        CUDA_TRY(cudaMemcpyAsync(staging[i], pinned[i], len, cudaMemcpyHostToDevice, m.st));
        CUDA_TRY(cudaEventRecord(done[i], m.st));
        *dev = staging[i];
        return {LLMB_OK, ""};
    }

    // loadMat / streamMat / streamMatNeox (gpu.go:287-391, fused.go:346-375):
    // one quantised [in, out] matrix into the tile layout, in pieces of at
    // most PieceSize bytes of whole tiles (whole heads when reordering).
    Error matrix(const std::string &name, int in, int out, QMat &q, int neox_hd = 0) {
        const Tensor *t = f.tensor(name);
        if (!t) return {LLMB_ERR_TENSOR, "llm: missing tensor " + name};
        if (t->dims.size() != 2 || (int64_t)t->dims[0] != in || (int64_t)t->dims[1] != out)
            return {LLMB_ERR_TENSOR, "llm: tensor " + name + " does not have the shape [" + std::to_string(in) + ", " +
                                         std::to_string(out) + "]"};
        if (t->type != GGML_Q4_0 && t->type != GGML_Q4_1 && t->type != GGML_Q8_0)
            return {LLMB_ERR_TENSOR, "llm: tensor " + name + " has ggml type " + std::to_string(t->type) +
                                         ", which has no GPU kernel (Q4_0, Q4_1, Q8_0)"};
        uint64_t be, bb;
        block_size(t->type, be, bb);
        q.type = (int)t->type;
        q.nb = in / 32;
        q.rows = (out + kTileRows - 1) / kTileRows * kTileRows;
        q.tile_bytes = tile_bytes_of(q.type, q.nb);
        Error err{LLMB_OK, ""};
        uint8_t *tiles = m.alloc<uint8_t>((size_t)q.tile_bytes * (q.rows / kTileRows), err);
        if (!tiles) return err;
        q.tiles = tiles;
        const uint64_t row_bytes = (uint64_t)q.nb * bb;
        const int align = neox_hd > 0 ? std::max(kTileRows, neox_hd) : kTileRows;
        if (neox_hd > 0 && (out % neox_hd != 0 || neox_hd % 2 != 0))
            return {LLMB_ERR_TENSOR, "llm: tensor " + name + ": rows are not whole heads"};
        int per = (int)(kPieceSize / row_bytes) / align * align;
        if (per < align) return {LLMB_ERR_TENSOR, "llm: tensor " + name + ": a row group exceeds the piece size"};
        for (int r0 = 0; r0 < out; r0 += per) {
            const int rows = std::min(per, out - r0);
            uint8_t *dev;
            if ((err = piece(f.data_offset + t->offset + (uint64_t)r0 * row_bytes, (uint64_t)rows * row_bytes, &dev))
                    .code)
                return err;
            launch_repack(dev, rows, q.nb, q.type, tiles, q.tile_bytes, r0, neox_hd, m.st);
            CUDA_TRY(cudaGetLastError());
        }
        return err;
    }

    // loadF32 (gpu.go:393-407); with neox_hd the entries are reordered like
    // the rows of their matrix (neoxRows, fused.go:336-344).
    Error vector(const std::string &name, int n, const float **out, int neox_hd = 0) {
        const Tensor *t = f.tensor(name);
        if (!t || t->type != GGML_F32) return {LLMB_ERR_TENSOR, "llm: tensor " + name + " missing or not F32"};
        if (t->dims.size() != 1 || (int64_t)t->dims[0] != n)
            return {LLMB_ERR_TENSOR, "llm: tensor " + name + " does not have " + std::to_string(n) + " elements"};
        std::vector<float> v(n);
        if (read(f.data_offset + t->offset, v.data(), (uint64_t)n * 4) < (uint64_t)n * 4)
            return {LLMB_ERR_IO, "llm: short read of " + name};
        if (neox_hd > 0) {
            std::vector<float> p(n);
            for (int nr = 0; nr < n; nr++) {
                const int h = nr / neox_hd, kk = nr % neox_hd;
                p[nr] = v[h * neox_hd + kk / 2 + (kk % 2) * (neox_hd / 2)];
            }
            v.swap(p);
        }
        Error err{LLMB_OK, ""};
        float *d = m.alloc<float>((size_t)n * 4, err);
        if (!d) return err;
        CUDA_TRY(cudaMemcpyAsync(d, v.data(), (size_t)n * 4, cudaMemcpyHostToDevice, m.st));
        CUDA_TRY(cudaStreamSynchronize(m.st));  // v is pageable and local
        *out = d;
        return err;
    }
};


// The largest tile (bytes) of the head and the layers' matrices.
static int max_tile_of(const DevModel &d, int layers) {
    int t = d.head.tile_bytes;
    for (int l = 0; l < layers; l++) {
        const Layer &L = d.layer[l];
        for (const QMat *q : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down}) t = std::max(t, q->tile_bytes);
    }
    return t;
}

Error open_model(Model &m, const ReadAt &read, uint64_t size, int ctx) {
    GgufFile f;
    std::string msg;
    GgufErr ge = gguf_parse(read, size, f, msg);
    if (ge != GgufErr::Ok)
        return {ge == GgufErr::Bound ? LLMB_ERR_BOUND : ge == GgufErr::Eof || ge == GgufErr::Io ? LLMB_ERR_IO
                                                                                                   : LLMB_ERR_FORMAT,
                msg};
    if (!config_from(f, m.cfg, msg)) return {LLMB_ERR_CONFIG, msg};
    Config &c = m.cfg;
    if (ctx <= 0 || ctx > c.ctx) ctx = c.ctx;  // gpu.go:470-472
    if (ctx <= 0) return {LLMB_ERR_CONFIG, "llm: the model has no context length"};
    c.ctx = ctx;
    if (c.layers > kMaxLayers) return {LLMB_ERR_CONFIG, "llm: more than 256 layers"};
    if (c.head_dim % 16 != 0 || c.embd % 32 != 0 || c.ff % 32 != 0)
        return {LLMB_ERR_CONFIG, "llm: the kernels need head_dim a multiple of 16 and embd, ff multiples of 32"};
    CUDA_TRY(cudaSetDevice(m.device));
    CUDA_TRY(cudaStreamCreateWithFlags(&m.st, cudaStreamNonBlocking));
    CUDA_TRY(cudaEventCreate(&m.ev0));
    CUDA_TRY(cudaEventCreate(&m.ev1));
    CUDA_TRY(cudaEventCreate(&m.ev2));
    CUDA_TRY(cudaEventCreate(&m.ev3));
    for (auto &l : m.lev)
        for (auto &e : l) CUDA_TRY(cudaEventCreate(&e));
    size_t free_b = 0, total_b = 0;
    CUDA_TRY(cudaMemGetInfo(&free_b, &total_b));
    const int64_t kb = g_memory_budget.load();
    m.budget = kb > 0 ? (uint64_t)kb : (uint64_t)free_b;
    m.pm = (int)std::clamp<int64_t>(g_prefill_batch.load(), 1, kMaxPrefill);

    const int kvd = c.kv_heads * c.head_dim, E = c.embd, F = c.ff;
    DevModel &d = m.hdm;
    d.embd = E, d.ff = F, d.heads = c.heads, d.kv_heads = c.kv_heads, d.head_dim = c.head_dim, d.kvd = kvd;
    d.vocab = c.vocab, d.ctx = ctx, d.layers = c.layers, d.eps = c.eps;
    d.scale = (float)(1.0 / std::sqrt((double)c.head_dim));  // cpu.go:304
    d.rope_neox = c.rope_neox;
    d.nchunk = (ctx + kAttnChunk - 1) / kAttnChunk;

    Shapes &s = m.sh;
    s.embd = E, s.ff = F, s.heads = c.heads, s.kv_heads = c.kv_heads, s.head_dim = c.head_dim, s.kvd = kvd;
    s.vocab = c.vocab, s.ctx = ctx, s.layers = c.layers, s.nchunk = d.nchunk;
    s.qkv_tiles = (E + 2 * kvd) / 8, s.o_tiles = E / 8, s.gu_tiles = F / 8, s.down_tiles = E / 8;
    s.head_tiles = (c.vocab + 7) / 8;
    int nsm = 0;
    CUDA_TRY(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, m.device));
    s.head_ctas = std::max(1, std::min(nsm * 2, (s.head_tiles + kWarps - 1) / kWarps));
    d.smem_vec = smem_vec_floats(s);
    CUDA_TRY(prepare_kernels(s));
    CUDA_TRY(prepare_products());
    m.persistent_ctas = nsm;

    Error err{LLMB_OK, ""};
    Loader ld{m, f, read};
    if ((err = ld.init()).code) return err;

    // token_embd: Q8_0 or Q4_0 gather (gpu.go:543-554)
    const Tensor *te = f.tensor("token_embd.weight");
    if (te->type != GGML_Q8_0 && te->type != GGML_Q4_0)
        return {LLMB_ERR_TENSOR, "llm: token_embd.weight must be Q8_0 or Q4_0"};
    if ((err = ld.matrix("token_embd.weight", E, c.vocab, d.embed)).code) return err;
    if ((err = ld.vector("output_norm.weight", E, &d.out_norm)).code) return err;
    if (c.tied_output) {
        d.head = d.embed;
    } else if ((err = ld.matrix("output.weight", E, c.vocab, d.head)).code) {
        return err;
    }
    const int neox = c.rope_neox ? c.head_dim : 0;  // fused.go:201-205
    for (int l = 0; l < c.layers; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        Layer &L = d.layer[l];
        if ((err = ld.vector(p + "attn_norm.weight", E, &L.attn_norm)).code) return err;
        if ((err = ld.matrix(p + "attn_q.weight", E, c.heads * c.head_dim, L.q, neox)).code) return err;
        if ((err = ld.matrix(p + "attn_k.weight", E, kvd, L.k, neox)).code) return err;
        if ((err = ld.matrix(p + "attn_v.weight", E, kvd, L.v)).code) return err;
        if (c.bias) {
            if ((err = ld.vector(p + "attn_q.bias", E, &L.bq, neox)).code) return err;
            if ((err = ld.vector(p + "attn_k.bias", kvd, &L.bk, neox)).code) return err;
            if ((err = ld.vector(p + "attn_v.bias", kvd, &L.bv)).code) return err;
        }
        if ((err = ld.matrix(p + "attn_output.weight", E, E, L.o)).code) return err;
        if ((err = ld.vector(p + "ffn_norm.weight", E, &L.ffn_norm)).code) return err;
        if ((err = ld.matrix(p + "ffn_gate.weight", E, F, L.gate)).code) return err;
        if ((err = ld.matrix(p + "ffn_up.weight", E, F, L.up)).code) return err;
        if ((err = ld.matrix(p + "ffn_down.weight", F, E, L.down)).code) return err;
        if (!(L.kv = m.alloc<float>((size_t)2 * ctx * kvd * 4, err))) return err;
    }
    // RoPE table in double precision (gpu.go:524-541)
    {
        const int hp = c.head_dim / 2;
        std::vector<float> cs((size_t)ctx * hp * 2);
        for (int pos = 0; pos < ctx; pos++)
            for (int i = 0; i < hp; i++) {
                const double theta =
                    (double)pos * std::pow((double)c.rope_base, -(double)(2 * i) / (double)c.head_dim);
                cs[((size_t)pos * hp + i) * 2] = (float)std::cos(theta);
                cs[((size_t)pos * hp + i) * 2 + 1] = (float)std::sin(theta);
            }
        float *dcs = m.alloc<float>(cs.size() * 4, err);
        if (!dcs) return err;
        CUDA_TRY(cudaMemcpyAsync(dcs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, m.st));
        CUDA_TRY(cudaStreamSynchronize(m.st));
        d.rope_cs = dcs;
    }
    // activations (gpu.go:508-523, fused.go:692-698)
    const int pm = kMaxPrefill;
    const int head_parts = std::max(s.head_ctas, m.persistent_ctas);
    if (!(d.x = m.alloc<float>((size_t)pm * E * 4, err))) return err;
    if (!(d.q = m.alloc<float>((size_t)pm * E * 4, err))) return err;
    if (!(d.att = m.alloc<float>((size_t)pm * E * 4, err))) return err;
    if (!(d.act = m.alloc<float>((size_t)pm * F * 4, err))) return err;
    if (!(d.logits = m.alloc<float>((size_t)c.vocab * 4, err))) return err;
    if (!(d.part_pv = m.alloc<float>((size_t)pm * c.heads * d.nchunk * c.head_dim * 4, err))) return err;
    if (!(d.part_ml = m.alloc<float2>((size_t)pm * c.heads * d.nchunk * 8, err))) return err;
    if (!(d.att_cnt = m.alloc<uint32_t>((size_t)pm * c.heads * 4, err))) return err;
    if (!(d.state = m.alloc<uint32_t>(8, err))) return err;
    if (!(d.tokens = m.alloc<int32_t>((size_t)(ctx + 1) * 4, err))) return err;
    if (!(d.am_part = m.alloc<float2>((size_t)head_parts * kMaxPrefill * 8, err))) return err;
    if (!(d.h = m.alloc<float>((size_t)pm * E * 4, err))) return err;
    if (!(d.ssq = m.alloc<float>((size_t)pm * kSsqTiles * 4, err))) return err;
    if (!(d.gam = m.alloc<float2>((size_t)pm * ((d.head.rows + 63) / 64) * 8, err))) return err;
    if (!(d.am_count = m.alloc<uint32_t>(kMaxPrefill * 4, err))) return err;
    if (!(d.err = m.alloc<int>(4, err))) return err;
    // the persistent decode kernel: tagged activations and its ring configuration
    if (!(d.ll_x = m.alloc<uint64_t>((size_t)E * 8, err))) return err;
    if (!(d.ll_q = m.alloc<uint64_t>((size_t)E * 8, err))) return err;
    if (!(d.ll_k = m.alloc<uint64_t>((size_t)kvd * 8, err))) return err;
    if (!(d.ll_v = m.alloc<uint64_t>((size_t)kvd * 8, err))) return err;
    if (!(d.ll_att = m.alloc<uint64_t>((size_t)E * 8, err))) return err;
    if (!(d.ll_act = m.alloc<uint64_t>((size_t)F * 8, err))) return err;
    if (!(d.ll_pv = m.alloc<uint64_t>((size_t)c.heads * d.nchunk * c.head_dim * 8, err))) return err;
    if (!(d.ll_ml = m.alloc<uint64_t>((size_t)c.heads * d.nchunk * 2 * 8, err))) return err;
    if (!(d.ll_am = m.alloc<uint64_t>((size_t)2 * m.persistent_ctas * 2 * 8, err))) return err;
    if (!(d.ll_epoch = m.alloc<uint32_t>(4, err))) return err;
    d.trace_events = c.layers * 5 + 2;
    if (g_decode_trace.load() &&
        !(d.trace = m.alloc<uint64_t>((size_t)m.persistent_ctas * d.trace_events * 4 * 8, err)))
        return err;
    {
        const int max_tile = max_tile_of(d, c.layers);
        const int T = F / 8, P = std::min(m.persistent_ctas, T);
        d.dec_gate_rows = (T + P - 1) / P * 8;
        const int Tq = (E + 2 * kvd) / 8, Pq = dec_qkv_ctas(Tq, m.persistent_ctas, c.heads);
        d.dec_qkv_rows = (Tq + Pq - 1) / Pq * 8;
        // the output and down shares reuse the gate buffer for their residual rows
        const int To = E / 8, Po = std::min(m.persistent_ctas, To);
        d.dec_gate_rows = std::max(d.dec_gate_rows, (To + Po - 1) / Po * 8);
        if (E > 1024) return {LLMB_ERR_CONFIG, "llm: the decode kernel supports embedding sizes up to 1024"};
        // the kernel splits each kind of matrix once per launch, from layer 0's shapes
        for (int l = 1; l < c.layers; l++) {
            const Layer &a = d.layer[0], &b = d.layer[l];
            const QMat *ma[] = {&a.q, &a.k, &a.v, &a.o, &a.gate, &a.up, &a.down};
            const QMat *mb[] = {&b.q, &b.k, &b.v, &b.o, &b.gate, &b.up, &b.down};
            for (int i = 0; i < 7; i++)
                if (ma[i]->rows != mb[i]->rows || ma[i]->nb != mb[i]->nb)
                    return {LLMB_ERR_CONFIG, "llm: the decode kernel needs every layer to have layer 0's shapes"};
        }
        if (c.head_dim != 64 && c.head_dim != 128)
            return {LLMB_ERR_CONFIG, "llm: the decode kernel supports head sizes 64 and 128"};
        m.dec = decode_config(s, max_tile, d.head.tile_bytes, d.dec_gate_rows, d.dec_qkv_rows, 0,
                              (int)g_attn_positions.load());
        d.dec_chunk = m.dec.chunk;
        if (c.layers > kMaxDecLayers) return {LLMB_ERR_CONFIG, "llm: the decode kernel supports up to 64 layers"};
        if (m.dec.nslots < 2 || decode2_ctas_per_sm(m.dec) < 1)
            return {LLMB_ERR_CONFIG, "llm: the decode kernel does not fit an SM (tiles of " + std::to_string(max_tile) +
                                         " bytes)"};
    }
    FeedUnit *plan = nullptr;
    int *plan_count = nullptr;
    if (!(plan = m.alloc<FeedUnit>((size_t)m.persistent_ctas * kMaxFeedPlan * sizeof(FeedUnit), err))) return err;
    if (!(plan_count = m.alloc<int>((size_t)m.persistent_ctas * 4, err))) return err;
    d.feed_plan = plan, d.feed_count = plan_count;
    if (!(m.dm = m.alloc<DevModel>(sizeof(DevModel), err))) return err;
    d.layers_g = m.dm->layer;  // the device address of the array (nothing is read here)
    CUDA_TRY(cudaMemcpyAsync(m.dm, &d, sizeof(DevModel), cudaMemcpyHostToDevice, m.st));
    m.dp = std::make_unique<DecParams>();
    static_cast<ModelHeader &>(*m.dp) = static_cast<const ModelHeader &>(d);
    for (int l = 0; l < c.layers; l++) m.dp->layer[l] = d.layer[l];
    {
        // the persistent kernel's weight stream, listed once: its length per CTA sizes the kernel's shared memory
        CUDA_TRY(launch_feed_plan(*m.dp, m.dec.slot_bytes, plan, plan_count, m.persistent_ctas, m.st));
        std::vector<int> counts(m.persistent_ctas);
        CUDA_TRY(cudaMemcpyAsync(counts.data(), plan_count, counts.size() * 4, cudaMemcpyDeviceToHost, m.st));
        CUDA_TRY(cudaStreamSynchronize(m.st));
        int mx = 0;
        for (int v : counts) {
            if (v < 0) return {LLMB_ERR_CONFIG, "llm: the decode kernel's weight stream exceeds its plan"};
            mx = std::max(mx, v);
        }
        m.dp->feed_max = mx;
        const DecConfig full = decode_config(s, max_tile_of(d, c.layers), d.head.tile_bytes, d.dec_gate_rows,
                                             d.dec_qkv_rows, mx, (int)g_attn_positions.load());
        if (full.nslots != m.dec.nslots || full.slot_bytes != m.dec.slot_bytes || full.smem > 232448 ||
            decode2_ctas_per_sm(full) < 1)
            return {LLMB_ERR_CONFIG, "llm: the decode kernel does not fit an SM with its weight plan"};
        m.dec = full;
        m.dp->dec_chunk = full.chunk;
    }
    CUDA_TRY(cudaHostAlloc(&m.h_tokens, (size_t)(ctx + 2 * kMaxDecodeBatch + 1) * 4, cudaHostAllocDefault));
    CUDA_TRY(cudaHostAlloc(&m.h_state, 16, cudaHostAllocDefault));
    CUDA_TRY(cudaHostAlloc(&m.h_err, 4 * 4, cudaHostAllocDefault));  // [0] checks; [1 + slot] a decode launch's
    std::memset(m.h_err, 0, 4 * 4);
    CUDA_TRY(cudaStreamSynchronize(m.st));
    m.stats.submits++;
    return err;
}

// ------------------------------------------------------------- running --

cudaError_t reset_tags(Model &m);

// Reads the device error word (after everything queued on the stream).  On an
// error it is cleared, and so are the persistent kernel's tagged buffers: a
// launch that gave up leaves words whose tags the next launch would reuse
// (the epoch counter advances only when a launch completes).
// The device error word, already copied to m.h_err by a synchronised stream: a
// device error becomes LLMB_ERR_DEVICE, after the word, the tags and the
// token count of the persistent kernel are reset.
Error device_status(Model &m) {
    if (*m.h_err != 0) {
        const int e = *m.h_err;
        *m.h_err = 0;
        cudaMemsetAsync(m.hdm.err, 0, 4, m.st);
        reset_tags(m);
        m.ll_tokens = 0;
        cudaStreamSynchronize(m.st);
        const char *what = e == DEV_BARRIER_TIMEOUT ? "a grid barrier of the decode kernel timed out"
                           : e == DEV_TAG_TIMEOUT   ? "an activation of the decode kernel did not arrive in time"
                           : e == DEV_RING_TIMEOUT  ? "a weight slot of the decode kernel timed out"
                           : e == DEV_MMA_TIMEOUT   ? "a tensor-core product did not complete in time"
                                                    : "a token past the context";
        return {LLMB_ERR_DEVICE, std::string("llm: ") + what};
    }
    return {LLMB_OK, ""};
}

Error check_device(Model &m) {
    CUDA_TRY(cudaMemcpyAsync(m.h_err, m.hdm.err, 4, cudaMemcpyDeviceToHost, m.st));
    CUDA_TRY(cudaStreamSynchronize(m.st));
    return device_status(m);
}

int layers_to_run(const Model &m) {
    if (m.layers_run == 0 || m.layers_run >= m.cfg.layers) return m.cfg.layers;
    return std::max(m.layers_run, 0);
}

// begin (gpu.go:838-847): state = {0, 0}, tokens[0:] = prompt.
Error begin(Model &m, const int32_t *prompt, int n) {
    std::memcpy(m.h_tokens, prompt, (size_t)n * 4);
    m.h_state[0] = m.h_state[1] = 0;
    CUDA_TRY(cudaMemcpyAsync(m.hdm.tokens, m.h_tokens, (size_t)n * 4, cudaMemcpyHostToDevice, m.st));
    CUDA_TRY(cudaMemcpyAsync(m.hdm.state, m.h_state, 8, cudaMemcpyHostToDevice, m.st));
    return {LLMB_OK, ""};
}

// The embedding and nl layers of cnt tokens through the chunked products,
// as a CUDA graph captured on first use (the kernels read positions, tokens
// and KV slots from device memory, so one graph serves every call).
Error run_layers_mm(Model &m, int cnt, int nl, const TokBatch *tb) {
    const bool tensor = g_prefill_mode.load() == 0;
    const int64_t key = (((int64_t)cnt * 2 + (tb ? 1 : 0)) * 1024 + nl) * 2 + (tensor ? 1 : 0);
    auto it = m.graphs.find(key);
    if (it == m.graphs.end()) {
        CUDA_TRY(cudaStreamBeginCapture(m.st, cudaStreamCaptureModeThreadLocal));
        launch_embed(m.dm, m.sh, cnt, m.st, tb);
        cudaError_t e = cudaGetLastError();
        for (int l = 0; l < nl && e == cudaSuccess; l++)
            e = launch_layer_mm(m.dm, m.hdm, m.sh, l, cnt, m.persistent_ctas, m.st, tb, tensor);
        cudaGraph_t g = nullptr;
        const cudaError_t e2 = cudaStreamEndCapture(m.st, &g);
        if (e == cudaSuccess) e = e2;
        cudaGraphExec_t ex = nullptr;
        if (e == cudaSuccess) e = cudaGraphInstantiate(&ex, g, 0);
        if (g) cudaGraphDestroy(g);
        CUDA_TRY(e);
        it = m.graphs.emplace(key, ex).first;
    }
    CUDA_TRY(cudaGraphLaunch(it->second, m.st));
    return {LLMB_OK, ""};
}

// prefill (gpu.go:853-900) over chunks of pm tokens (chunk, fused.go:294-320):
// the last chunk's last token goes through the head, which samples tokens[n].
Error prefill(Model &m, int n) {
    const int nl = layers_to_run(m);
    const bool head = nl == m.cfg.layers;
    for (int a = 0; a < n; a += m.pm) {
        const int cnt = std::min(m.pm, n - a);
        const bool last = a + cnt == n;
        if (g_prefill_mode.load() != 1) {
            Error e = run_layers_mm(m, cnt, nl, nullptr);
            if (e.code) return e;
            m.stats.dispatches += 1 + (g_prefill_mode.load() == 0 ? 5 : 7) * nl;
        } else {
            if (nl == 0) {
                launch_embed(m.dm, m.sh, cnt, m.st);
                m.stats.dispatches++;
            }
            for (int l = 0; l < nl; l++) launch_layer(m.dm, m.sh, l, cnt, m.st);
            m.stats.dispatches += 5 * nl;
        }
        if (last && head) launch_head(m.dm, m.sh, cnt - 1, cnt, m.st);
        else launch_advance(m.dm, cnt, m.st);
        m.stats.dispatches++;
        m.stats.submits++;
        CUDA_TRY(cudaGetLastError());
    }
    return {LLMB_OK, ""};
}

// Zeroes the persistent kernel's tagged exchange buffers and its epoch counter
// (stream-ordered after every launch before it).
cudaError_t reset_tags(Model &m) {
    const DevModel &d = m.hdm;
    const int E = m.cfg.embd, F = m.cfg.ff, kvd = d.kvd;
    const std::pair<void *, size_t> bufs[] = {
        {d.ll_x, (size_t)E * 8}, {d.ll_q, (size_t)E * 8}, {d.ll_k, (size_t)kvd * 8}, {d.ll_v, (size_t)kvd * 8},
        {d.ll_att, (size_t)E * 8}, {d.ll_act, (size_t)F * 8},
        {d.ll_pv, (size_t)m.cfg.heads * d.nchunk * m.cfg.head_dim * 8}, {d.ll_ml, (size_t)m.cfg.heads * d.nchunk * 2 * 8},
        {d.ll_am, (size_t)2 * m.persistent_ctas * 2 * 8}, {d.ll_epoch, 4}};
    for (const auto &b : bufs) {
        const cudaError_t e = cudaMemsetAsync(b.first, 0, b.second, m.st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// cnt decode tokens: the persistent kernel (one launch) or the per-phase kernels.
Error decode(Model &m, int cnt) {
    if (g_decode_mode.load() == 0) {
        // The exchange tags are 32-bit, epoch * 8 (layers + 1) + phase: before they would wrap (about
        // 17M tokens for 30 layers), clear the tagged buffers and restart the epoch, so that no stale
        // word can carry a live tag.
        const int64_t per_token = 8 * ((int64_t)m.cfg.layers + 1), forced = g_tag_reset.load();
        if ((m.ll_tokens + cnt + 2) * per_token >= (int64_t)UINT32_MAX || (forced > 0 && m.ll_tokens >= forced)) {
            CUDA_TRY(reset_tags(m));
            m.ll_tokens = 0;
        }
        m.dp->wait_ns = (uint64_t)g_wait_limit_us.load() * 1000u;
        m.dp->drop_step = (int)g_drop_publish.load();
        CUDA_TRY(launch_decode2(*m.dp, m.dec, cnt, m.persistent_ctas, m.st));
        m.ll_tokens += cnt;
        m.stats.dispatches++;
    } else {
        for (int j = 0; j < cnt; j++) {
            for (int l = 0; l < m.cfg.layers; l++) launch_layer(m.dm, m.sh, l, 1, m.st);
            launch_head(m.dm, m.sh, 0, 1, m.st);
            m.stats.dispatches += 5 * m.cfg.layers + 1;
        }
        CUDA_TRY(cudaGetLastError());
    }
    m.stats.submits++;
    return {LLMB_OK, ""};
}

Error check_prompt(const Model &m, const int32_t *prompt, int n) {
    if (n <= 0 || !prompt) return {LLMB_ERR_ARG, "llm: empty prompt"};  // gpu.go:854-856
    for (int i = 0; i < n; i++)
        if (prompt[i] < 0 || prompt[i] >= m.cfg.vocab)
            return {LLMB_ERR_ARG, "llm: token id " + std::to_string(prompt[i]) + " is outside the vocabulary"};
    return {LLMB_OK, ""};
}

// Generate, gpu.go:941-1014.  The decode loop keeps up to two launches in
// flight: launch k+1 is queued (its input token is already on the device)
// before the tokens of launch k are read back, so the GPU does not wait for
// the host between launches.
Error generate(Model &m, const int32_t *prompt, int np, int n, int32_t eos, llmb_emit_fn emit, void *user,
               int32_t *out_tokens, int *n_out, llmb_timing *tm_out) {
    llmb_timing tm{};
    if (n_out) *n_out = 0;
    if (n < 0) return {LLMB_ERR_ARG, "llm: negative token count"};
    if ((int64_t)np + n > m.cfg.ctx)
        return {LLMB_ERR_CONTEXT, "llm: prompt of " + std::to_string(np) + " tokens and " + std::to_string(n) +
                                      " new tokens exceed the context of " + std::to_string(m.cfg.ctx)};
    Error err = check_prompt(m, prompt, np);
    if (err.code) return err;
    if (layers_to_run(m) != m.cfg.layers)
        return {LLMB_ERR_ARG, "llm: Generate needs every layer (Layers is a PrefillLogits/Peek debugging aid)"};
    const int64_t s0 = m.stats.submits, d0 = m.stats.dispatches;
    const double t0 = now_ms();
    CUDA_TRY(cudaEventRecord(m.ev0, m.st));
    if ((err = begin(m, prompt, np)).code) return err;
    if ((err = prefill(m, np)).code) return err;
    CUDA_TRY(cudaEventRecord(m.ev1, m.st));
    // the first sampled token comes back with the prefill (gpu.go:954-958)
    int32_t *slot[2] = {m.h_tokens, m.h_tokens + kMaxDecodeBatch};
    CUDA_TRY(cudaMemcpyAsync(slot[0], m.hdm.tokens + np, 4, cudaMemcpyDeviceToHost, m.st));
    CUDA_TRY(cudaMemcpyAsync(m.h_err, m.hdm.err, 4, cudaMemcpyDeviceToHost, m.st));
    CUDA_TRY(cudaStreamSynchronize(m.st));
    if ((err = device_status(m)).code) return err;
    tm.prefill_ms = now_ms() - t0;
    tm.prompt_tokens = np;
    const double t1 = now_ms();
    const int batch = (int)std::clamp<int64_t>(g_decode_batch.load(), 1, kMaxDecodeBatch);
    struct Launch {
        int cnt, slot;
    };
    Launch q[2];
    int qh = 0, qn = 0;                 // ring of launches whose tokens are not read yet
    int issued = 1, produced = 0, k = 0;  // tokens launched (the prefill sampled the first), emitted
    int pending = 1, pending_slot = 0;    // tokens of the oldest read-back already waited for
    bool any_decode = false;
    bool stop = false;
    while (!stop) {
        // emit what the last wait brought back
        for (int j = 0; j < pending && produced < n; j++) {
            const int32_t tok = slot[pending_slot][j];
            if (tok == eos) {  // the tokens computed past it are dropped
                stop = true;
                break;
            }
            if (out_tokens) out_tokens[produced] = tok;
            tm.generated++;
            produced++;
            m.stats.tokens++;
            if (emit && !emit(user, tok)) {
                stop = true;
                break;
            }
        }
        if (stop || produced >= n) break;
        // keep two launches in flight
        while (qn < 2 && issued < n) {
            const int cnt = std::min(batch, n - issued);
            const int sl = (pending_slot + 1 + qn) & 1;
            const double ta = now_ms();
            CUDA_TRY(cudaEventRecord(m.lev[k & 3][0], m.st));
            if (!any_decode) {
                CUDA_TRY(cudaEventRecord(m.ev2, m.st));
                any_decode = true;
            }
            if ((err = decode(m, cnt)).code) return err;
            CUDA_TRY(cudaEventRecord(m.lev[k & 3][1], m.st));
            CUDA_TRY(cudaMemcpyAsync(slot[sl], m.hdm.tokens + np + issued, (size_t)cnt * 4, cudaMemcpyDeviceToHost,
                                     m.st));
            // the device error word after this launch, read back with its tokens (no stream-wide wait, so
            // the other launch stays in flight)
            CUDA_TRY(cudaMemcpyAsync(m.h_err + 1 + sl, m.hdm.err, 4, cudaMemcpyDeviceToHost, m.st));
            CUDA_TRY(cudaEventRecord(m.lev[k & 3][2], m.st));
            tm.record_ms += now_ms() - ta;
            q[(qh + qn) & 1] = {cnt, sl};
            m.lk[(qh + qn) & 1] = k & 3;
            qn++, k++, issued += cnt;
        }
        if (qn == 0) break;
        // wait for the oldest launch's tokens
        const double tb = now_ms();
        const int li = m.lk[qh];
        CUDA_TRY(cudaEventSynchronize(m.lev[li][2]));
        tm.submit_ms += now_ms() - tb;
        float kms = 0;
        cudaEventElapsedTime(&kms, m.lev[li][0], m.lev[li][1]);
        tm.decode_kernel_ms += kms;
        tm.decode_launches++;
        if (m.h_err[1 + q[qh].slot] != 0) {  // a device error: the full check resets the state and reports it
            m.h_err[1 + q[qh].slot] = 0;
            if ((err = check_device(m)).code) return err;
        }
        pending = q[qh].cnt, pending_slot = q[qh].slot;
        qh = (qh + 1) & 1, qn--;
    }
    CUDA_TRY(cudaStreamSynchronize(m.st));  // launches queued past a stop
    if ((err = check_device(m)).code) return err;
    CUDA_TRY(cudaEventRecord(m.ev3, m.st));
    CUDA_TRY(cudaEventSynchronize(m.ev3));
    tm.decode_ms = now_ms() - t1;
    float a = 0, b = 0;
    cudaEventElapsedTime(&a, m.ev0, m.ev1);
    if (any_decode) cudaEventElapsedTime(&b, m.ev2, m.ev3);
    tm.gpu_prefill_ms = a, tm.gpu_decode_ms = b;
    tm.submits = m.stats.submits - s0, tm.dispatches = m.stats.dispatches - d0;
    if (n_out) *n_out = produced;
    if (tm_out) *tm_out = tm;
    return {LLMB_OK, ""};
}

// Multi-stream generation (config 5): nseq independent greedy sequences on
// one model, each with its own KV slot in an arena.  The prompt tokens of all
// sequences are packed into batches of up to kMaxPrefill tokens, each
// sequence's in order (a token's attention reads KV rows written by an
// earlier launch, or by the QKV launch of its own batch, which runs before
// the batch's attention launch); the last prompt token of a sequence goes
// through the batch head.  Then every decode step runs one token of each
// unfinished sequence, kMaxPrefill per launch set.  Per sequence the
// semantics are Generate's (gpu.go:946-1014): eos stops it and is not
// emitted, n tokens at most.
Error ensure_batch(Model &m, int nseq) {
    Error err{LLMB_OK, ""};
    if (!m.tb) {
        if (!(m.tb = m.alloc<TokBatch>(sizeof(TokBatch), err))) return err;
        CUDA_TRY(cudaHostAlloc(&m.h_tb, sizeof(TokBatch), cudaHostAllocDefault));
        std::memset(m.h_tb, 0, sizeof(TokBatch));
    }
    if (m.bkv_slots < nseq) {
        if (m.bkv) m.release(m.bkv), m.bkv = nullptr, m.bkv_slots = 0;
        const size_t per = (size_t)m.cfg.layers * 2 * m.cfg.ctx * m.hdm.kvd;
        if (!(m.bkv = m.alloc<float>((size_t)nseq * per * 4, err))) return err;
        m.bkv_slots = nseq;
    }
    m.h_tb->kv = m.bkv;
    m.h_tb->layers = m.cfg.layers;
    return err;
}

// Runs the rows staged in m.h_tb (cnt tokens, nh of them through the head)
// and returns the head's tokens in m.h_tb->out.
Error run_batch(Model &m, int cnt, int nh) {
    CUDA_TRY(cudaMemcpyAsync(m.tb, m.h_tb, sizeof(TokBatch), cudaMemcpyHostToDevice, m.st));
    const bool mm = g_prefill_mode.load() != 1;
    if (mm) {
        Error e = run_layers_mm(m, cnt, m.cfg.layers, m.tb);
        if (e.code) return e;
        m.stats.dispatches += 1 + (g_prefill_mode.load() == 0 ? 5 : 7) * m.cfg.layers;
    } else {
        for (int l = 0; l < m.cfg.layers; l++) launch_layer(m.dm, m.sh, l, cnt, m.st, m.tb);
        m.stats.dispatches += 5 * m.cfg.layers;
    }
    if (nh > 0) {
        if (mm)
            CUDA_TRY(launch_head_mm(m.dm, m.hdm, m.sh, m.tb, m.tb->head_rows, nh, m.persistent_ctas, m.st,
                                    g_prefill_mode.load() == 0));
        else launch_head_batch(m.dm, m.sh, m.tb, nh, m.st);
        m.stats.dispatches += mm ? 3 : 1;
        CUDA_TRY(cudaMemcpyAsync(m.h_tb->out, m.tb->out, (size_t)nh * 4, cudaMemcpyDeviceToHost, m.st));
    }
    // the error word with the tokens: one synchronisation per batch
    CUDA_TRY(cudaMemcpyAsync(m.h_err, m.hdm.err, 4, cudaMemcpyDeviceToHost, m.st));
    CUDA_TRY(cudaGetLastError());
    m.stats.submits++;
    CUDA_TRY(cudaStreamSynchronize(m.st));
    return device_status(m);
}

Error generate_batch(Model &m, const int32_t *prompts, const int *lens, int nseq, int n, int32_t eos, int32_t *out,
                     int *n_out, llmb_timing *tm_out) {
    llmb_timing tm{};
    if (nseq <= 0 || !prompts || !lens) return {LLMB_ERR_ARG, "llm: no sequences"};
    if (n < 0) return {LLMB_ERR_ARG, "llm: negative token count"};
    if (n > 0 && !out) return {LLMB_ERR_ARG, "llm: no output buffer"};
    if (layers_to_run(m) != m.cfg.layers) return {LLMB_ERR_ARG, "llm: generation needs every layer"};
    std::vector<int64_t> off(nseq + 1, 0);
    for (int s = 0; s < nseq; s++) {
        if ((int64_t)lens[s] + n > m.cfg.ctx)
            return {LLMB_ERR_CONTEXT, "llm: sequence " + std::to_string(s) + ": prompt of " + std::to_string(lens[s]) +
                                          " tokens and " + std::to_string(n) + " new tokens exceed the context of " +
                                          std::to_string(m.cfg.ctx)};
        Error err = check_prompt(m, prompts + off[s], lens[s]);
        if (err.code) return err;
        off[s + 1] = off[s] + lens[s];
    }
    if (n_out) std::fill(n_out, n_out + nseq, 0);
    Error err = ensure_batch(m, nseq);
    if (err.code) return err;
    const int64_t s0 = m.stats.submits, d0 = m.stats.dispatches;
    const double t0 = now_ms();
    CUDA_TRY(cudaEventRecord(m.ev0, m.st));
    std::vector<int> gen(nseq, 0), last(nseq, 0);
    std::vector<char> done(nseq, n == 0);
    auto take = [&](int s, int tok) {  // a sampled token of sequence s
        if (done[s]) return;
        if (tok == eos) {
            done[s] = 1;
            return;
        }
        out[(size_t)s * n + gen[s]] = tok;
        last[s] = tok;
        if (++gen[s] >= n) done[s] = 1;
        tm.generated++;
        m.stats.tokens++;
    };
    // prompts, packed
    TokBatch &hb = *m.h_tb;
    int cnt = 0, nh = 0;
    std::vector<int> head_seq(kMaxPrefill);
    for (int s = 0; s < nseq; s++) {
        for (int i = 0; i < lens[s]; i++) {
            hb.pos[cnt] = i, hb.slot[cnt] = s, hb.tok[cnt] = prompts[off[s] + i];
            if (i == lens[s] - 1) hb.head_rows[nh] = cnt, head_seq[nh++] = s;
            if (++cnt == kMaxPrefill) {
                if ((err = run_batch(m, cnt, nh)).code) return err;
                for (int j = 0; j < nh; j++) take(head_seq[j], hb.out[j]);
                cnt = nh = 0;
            }
        }
        tm.prompt_tokens += lens[s];
    }
    if (cnt > 0) {
        if ((err = run_batch(m, cnt, nh)).code) return err;
        for (int j = 0; j < nh; j++) take(head_seq[j], hb.out[j]);
    }
    CUDA_TRY(cudaEventRecord(m.ev1, m.st));
    tm.prefill_ms = now_ms() - t0;
    const double t1 = now_ms();
    CUDA_TRY(cudaEventRecord(m.ev2, m.st));
    // decode steps: one token of every unfinished sequence
    std::vector<int> rows;
    for (;;) {
        rows.clear();
        for (int s = 0; s < nseq; s++)
            if (!done[s]) rows.push_back(s);
        if (rows.empty()) break;
        for (size_t a = 0; a < rows.size(); a += kMaxPrefill) {
            const int c = (int)std::min<size_t>(kMaxPrefill, rows.size() - a);
            for (int r = 0; r < c; r++) {
                const int s = rows[a + r];
                hb.pos[r] = lens[s] + gen[s] - 1, hb.slot[r] = s, hb.tok[r] = last[s], hb.head_rows[r] = r;
            }
            if ((err = run_batch(m, c, c)).code) return err;
            for (int r = 0; r < c; r++) take(rows[a + r], hb.out[r]);
        }
    }
    CUDA_TRY(cudaEventRecord(m.ev3, m.st));
    CUDA_TRY(cudaEventSynchronize(m.ev3));
    tm.decode_ms = now_ms() - t1;
    float a = 0, b = 0;
    cudaEventElapsedTime(&a, m.ev0, m.ev1);
    cudaEventElapsedTime(&b, m.ev2, m.ev3);
    tm.gpu_prefill_ms = a, tm.gpu_decode_ms = b;
    tm.submits = m.stats.submits - s0, tm.dispatches = m.stats.dispatches - d0;
    if (n_out)
        for (int s = 0; s < nseq; s++) n_out[s] = gen[s];
    if (tm_out) *tm_out = tm;
    return {LLMB_OK, ""};
}

Error prefill_logits(Model &m, const int32_t *prompt, int np, float *logits) {
    if (np >= m.cfg.ctx) return {LLMB_ERR_CONTEXT, "llm: prompt longer than the context"};  // gpu.go:905-907
    Error err = check_prompt(m, prompt, np);
    if (err.code) return err;
    if ((err = begin(m, prompt, np)).code) return err;
    if ((err = prefill(m, np)).code) return err;
    if (logits) CUDA_TRY(cudaMemcpyAsync(logits, m.hdm.logits, (size_t)m.cfg.vocab * 4, cudaMemcpyDeviceToHost, m.st));
    CUDA_TRY(cudaStreamSynchronize(m.st));
    return check_device(m);
}

Error generate_logits(Model &m, const int32_t *prompt, int np, int n, int32_t *toks, float *step_logits) {
    if (n <= 0) return {LLMB_ERR_ARG, "llm: no tokens to generate"};
    if ((int64_t)np + n > m.cfg.ctx) return {LLMB_ERR_CONTEXT, "llm: prompt and new tokens exceed the context"};
    if (layers_to_run(m) != m.cfg.layers) return {LLMB_ERR_ARG, "llm: generation needs every layer"};
    Error err = prefill_logits(m, prompt, np, step_logits);
    if (err.code) return err;
    for (int i = 0; i < n; i++) {
        if (i > 0) {
            if ((err = decode(m, 1)).code) return err;
            if (step_logits)
                CUDA_TRY(cudaMemcpyAsync(step_logits + (size_t)i * m.cfg.vocab, m.hdm.logits, (size_t)m.cfg.vocab * 4,
                                         cudaMemcpyDeviceToHost, m.st));
        }
        CUDA_TRY(cudaMemcpyAsync(toks + i, m.hdm.tokens + np + i, 4, cudaMemcpyDeviceToHost, m.st));
        CUDA_TRY(cudaStreamSynchronize(m.st));
        if ((err = check_device(m)).code) return err;
    }
    return err;
}

// Peek, gpu.go:1016-1043.
Error peek(Model &m, const char *name, float *out, int n) {
    const DevModel &d = m.hdm;
    const void *p = nullptr;
    size_t words = 0;
    const std::string s = name ? name : "";
    const size_t pm = kMaxPrefill;
    if (s == "x") p = d.x, words = pm * d.embd;
    else if (s == "q") p = d.q, words = pm * d.embd;
    else if (s == "att") p = d.att, words = pm * d.embd;
    else if (s == "gate") p = d.act, words = pm * d.ff;
    else if (s == "logits") p = d.logits, words = d.vocab;
    else if (s == "state") p = d.state, words = 2;
    else if (s == "tokens") p = d.tokens, words = (size_t)d.ctx + 1;
    else if (s == "trace" && d.trace) p = d.trace, words = (size_t)m.persistent_ctas * d.trace_events * 4 * 2;
    else if (s.rfind("kvblk.", 0) == 0) {
        int l = -1;
        if (std::sscanf(s.c_str(), "kvblk.%d.", &l) == 1 && l >= 0 && l < d.layers)
            p = d.layer[l].kv, words = (size_t)2 * d.ctx * d.kvd;
    }
    if (!p) return {LLMB_ERR_ARG, "llm: no buffer \"" + s + "\""};
    if (n < 0 || (size_t)n > words) return {LLMB_ERR_ARG, "llm: buffer \"" + s + "\" has " + std::to_string(words) + " words"};
    CUDA_TRY(cudaMemcpyAsync(out, p, (size_t)n * 4, cudaMemcpyDeviceToHost, m.st));
    CUDA_TRY(cudaStreamSynchronize(m.st));
    m.stats.submits++;
    return {LLMB_OK, ""};
}

int fail(Model *m, const Error &e) {
    if (m) m->last_error = e.msg;
    return e.code;
}

int open_common(const ReadAt &read, uint64_t size, int ctx, int device, llmb_model **out) {
    if (!out) return LLMB_ERR_ARG;
    *out = nullptr;
    auto m = std::make_unique<Model>();
    m->device = device;
    Error e;
    try {
        e = open_model(*m, read, size, ctx);
    } catch (const std::exception &ex) {
        e = {LLMB_ERR_MEMORY, std::string("llm: ") + ex.what()};
    }
    if (e.code) {
        t_open_error = e.msg;
        return e.code;
    }
    t_open_error.clear();
    *out = reinterpret_cast<llmb_model *>(m.release());
    return LLMB_OK;
}

inline Model *M(llmb_model *m) { return reinterpret_cast<Model *>(m); }
inline const Model *M(const llmb_model *m) { return reinterpret_cast<const Model *>(m); }

}  // namespace
}  // namespace llmb

using namespace llmb;

extern "C" {

int llmb_open(const char *path, int ctx, int device, llmb_model **out) {
    if (!path) return LLMB_ERR_ARG;
    int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        t_open_error = std::string("llm: open ") + path + ": " + std::strerror(errno);
        return LLMB_ERR_IO;
    }
    struct stat stt;
    fstat(fd, &stt);
    ReadAt read = [fd](uint64_t off, void *buf, uint64_t len) -> uint64_t {
        uint64_t got = 0;
        while (got < len) {
            ssize_t r = ::pread(fd, (char *)buf + got, len - got, (off_t)(off + got));
            if (r <= 0) break;
            got += (uint64_t)r;
        }
        return got;
    };
    int rc = open_common(read, (uint64_t)stt.st_size, ctx, device, out);
    ::close(fd);
    return rc;
}

int llmb_open_reader(llmb_read_fn fn, void *user, uint64_t size, int ctx, int device, llmb_model **out) {
    if (!fn) return LLMB_ERR_ARG;
    ReadAt read = [fn, user](uint64_t off, void *buf, uint64_t len) -> uint64_t {
        return fn(user, off, buf, len) == 0 ? len : 0;
    };
    return open_common(read, size, ctx, device, out);
}

void llmb_close(llmb_model *m) {
    if (!m) return;
    cudaSetDevice(M(m)->device);
    delete M(m);
}

const char *llmb_last_error(const llmb_model *m) {
    if (!m) return t_open_error.c_str();
    return M(m)->last_error.c_str();
}

int llmb_get_config(const llmb_model *mp, llmb_config *out) {
    if (!mp || !out) return LLMB_ERR_ARG;
    const Config &c = M(mp)->cfg;
    *out = llmb_config{};
    out->layers = c.layers, out->embd = c.embd, out->ff = c.ff, out->heads = c.heads, out->kv_heads = c.kv_heads;
    out->head_dim = c.head_dim, out->vocab = c.vocab, out->ctx = c.ctx, out->rope_base = c.rope_base, out->eps = c.eps;
    out->rope_neox = c.rope_neox, out->bias = c.bias, out->tied_output = c.tied_output;
    std::strncpy(out->arch, c.arch.c_str(), sizeof(out->arch) - 1);
    return LLMB_OK;
}

uint64_t llmb_memory_used(const llmb_model *m) { return m ? M(m)->used : 0; }

int llmb_get_stats(const llmb_model *m, llmb_stats *out) {
    if (!m || !out) return LLMB_ERR_ARG;
    *out = M(m)->stats;
    return LLMB_OK;
}

int llmb_generate(llmb_model *mp, const int32_t *prompt, int n_prompt, int n, int32_t eos, llmb_emit_fn emit,
                  void *user, int32_t *out_tokens, int *n_out, llmb_timing *tm) {
    if (!mp) return LLMB_ERR_ARG;
    Model *m = M(mp);
    cudaSetDevice(m->device);
    return fail(m, generate(*m, prompt, n_prompt, n, eos, emit, user, out_tokens, n_out, tm));
}

int llmb_generate_batch(llmb_model *mp, const int32_t *prompts, const int *prompt_lens, int n_seq, int n, int32_t eos,
                        int32_t *out_tokens, int *n_out, llmb_timing *tm) {
    if (!mp) return LLMB_ERR_ARG;
    Model *m = M(mp);
    cudaSetDevice(m->device);
    return fail(m, generate_batch(*m, prompts, prompt_lens, n_seq, n, eos, out_tokens, n_out, tm));
}

int llmb_prefill_logits(llmb_model *mp, const int32_t *prompt, int n_prompt, float *logits) {
    if (!mp) return LLMB_ERR_ARG;
    Model *m = M(mp);
    cudaSetDevice(m->device);
    return fail(m, prefill_logits(*m, prompt, n_prompt, logits));
}

int llmb_generate_logits(llmb_model *mp, const int32_t *prompt, int n_prompt, int n, int32_t *out_tokens,
                         float *step_logits) {
    if (!mp || !out_tokens) return LLMB_ERR_ARG;
    Model *m = M(mp);
    cudaSetDevice(m->device);
    return fail(m, generate_logits(*m, prompt, n_prompt, n, out_tokens, step_logits));
}

int llmb_peek(llmb_model *mp, const char *name, float *out, int n) {
    if (!mp || !out) return LLMB_ERR_ARG;
    Model *m = M(mp);
    cudaSetDevice(m->device);
    return fail(m, peek(*m, name, out, n));
}

int llmb_set_layers(llmb_model *mp, int layers) {
    if (!mp) return LLMB_ERR_ARG;
    M(mp)->layers_run = layers;
    return LLMB_OK;
}

int llmb_set_knob(const char *name, int64_t v) {
    if (!name) return LLMB_ERR_ARG;
    const std::string s = name;
    if (s == "decode_batch") g_decode_batch = std::clamp<int64_t>(v, 1, kMaxDecodeBatch);
    else if (s == "prefill_batch") g_prefill_batch = std::clamp<int64_t>(v, 1, kMaxPrefill);
    else if (s == "memory_budget") g_memory_budget = std::max<int64_t>(v, 0);
    else if (s == "decode_mode") g_decode_mode = v ? 1 : 0;
    else if (s == "decode_trace") g_decode_trace = v ? 1 : 0;
    else if (s == "prefill_mode") g_prefill_mode = std::clamp<int64_t>(v, 0, 2);
    else if (s == "tag_reset") g_tag_reset = v > 0 ? v : 0;
    else if (s == "attn_positions") g_attn_positions = v > 0 ? std::clamp<int64_t>(v, 64, 256) / 32 * 32 : 0;
    else if (s == "wait_limit_us") g_wait_limit_us = std::clamp<int64_t>(v, 0, 10000000);
    else if (s == "drop_publish") g_drop_publish = v >= 0 ? std::min<int64_t>(v, INT32_MAX) : -1;
    else return LLMB_ERR_ARG;
    return LLMB_OK;
}

int64_t llmb_get_knob(const char *name) {
    if (!name) return -1;
    const std::string s = name;
    if (s == "decode_batch") return g_decode_batch;
    if (s == "prefill_batch") return g_prefill_batch;
    if (s == "memory_budget") return g_memory_budget;
    if (s == "decode_mode") return g_decode_mode;
    if (s == "decode_trace") return g_decode_trace;
    if (s == "prefill_mode") return g_prefill_mode;
    if (s == "tag_reset") return g_tag_reset;
    if (s == "attn_positions") return g_attn_positions;
    if (s == "wait_limit_us") return g_wait_limit_us;
    if (s == "drop_publish") return g_drop_publish;
    return -1;
}

}  // extern "C"
