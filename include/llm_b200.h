/*
 * llm_b200.h -- the C ABI of the B200 forward pass for go-wasmcontainers/llm.
 *
 * A drop-in for the reference's GPU forward pass (gpu.go, fused.go,
 * kernels.go, kernels_fused.go): a Go host keeps its llm.GPU API and calls
 * these functions over cgo instead of recording WebGPU passes.  Each entry
 * point names the reference interface it replaces (file:line in the
 * reference repository).  Plain C types only; the library owns all device
 * memory, the caller owns every buffer it passes in.  No call aborts the
 * process: every failure is a status code with a message from
 * llmb_last_error.
 *
 * Threading (gpu.go:148,831): a model handle is used by one thread at a
 * time.  Several handles, one per device, may run concurrently from
 * separate threads; that is the multi-GPU mode (independent sequences).
 */
#ifndef LLM_B200_H
#define LLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define LLMB_API __attribute__((visibility("default")))
#else
#define LLMB_API
#endif

/* Status codes.  The reference returns Go error values; the classes below
 * follow its error sites. */
enum {
    LLMB_OK = 0,
    LLMB_ERR_ARG = 1,     /* a bad argument (empty prompt gpu.go:855, token id out of range) */
    LLMB_ERR_IO = 2,      /* reading the model file (gpu.go:365-367) */
    LLMB_ERR_FORMAT = 3,  /* GGUF header: gguf.ErrMagic, ErrVersion, ErrFormat (gguf/gguf.go:29-34) */
    LLMB_ERR_BOUND = 4,   /* GGUF header: gguf.ErrBound (gguf/gguf.go:32) */
    LLMB_ERR_CONFIG = 5,  /* ConfigFrom refusals (config.go:32-70) */
    LLMB_ERR_TENSOR = 6,  /* a missing tensor or a type without a kernel (gpu.go:300,326) */
    LLMB_ERR_MEMORY = 7,  /* the memory budget or a device allocation (gpu.go:175-177) */
    LLMB_ERR_CONTEXT = 8, /* prompt and new tokens exceed the context (gpu.go:948-950, 905-907) */
    LLMB_ERR_CUDA = 9,    /* a CUDA runtime error */
    LLMB_ERR_DEVICE = 10  /* a kernel reported an error (a bounded wait that gave up) */
};

typedef struct llmb_model llmb_model;

/* Config, config.go:11-23. */
typedef struct {
    int32_t layers, embd, ff, heads, kv_heads, head_dim, vocab, ctx;
    float rope_base, eps;
    int32_t rope_neox, bias, tied_output;
    char arch[16];
} llmb_config;

/* Stats, gpu.go:55-60.  A submit is one host->device launch group (one
 * CUDA graph launch or one prefill chunk); a dispatch is one kernel. */
typedef struct {
    int64_t submits, dispatches, tokens;
} llmb_stats;

/* Timing, gpu.go:929-939, plus device time from CUDA events on the model's
 * stream.  prefill_ms runs until the first sampled token is on the host;
 * decode_ms is the rest of the call.  gpu_decode_ms spans the first decode
 * launch to the end of the last; decode_kernel_ms sums the decode launches
 * alone (decode_launches of them). */
typedef struct {
    double prefill_ms, decode_ms;         /* wall clock, as time.Since in Generate */
    int32_t prompt_tokens, generated;
    int64_t submits, dispatches;
    double record_ms, submit_ms;          /* host time launching / waiting in decode */
    double gpu_prefill_ms, gpu_decode_ms; /* device time between CUDA events */
    double decode_kernel_ms;
    int64_t decode_launches;
} llmb_timing;

/* A reader of the model file: fill buf with len bytes at offset, return 0
 * on success.  Lets a Go host pass its io.ReaderAt (gpu.go:290,365). */
typedef int (*llmb_read_fn)(void *user, uint64_t offset, void *buf, uint64_t len);

/* Called with each generated token in order; return nonzero to go on, 0 to
 * stop (the emit callback of Generate, gpu.go:946,979). */
typedef int (*llmb_emit_fn)(void *user, int32_t token);

/* NewGPU, gpu.go:465-764.  Parses the GGUF header (gguf.Parse,
 * gguf/gguf.go:292), checks the configuration (ConfigFrom, config.go:29),
 * allocates every device buffer, builds the RoPE table in double precision
 * (gpu.go:524-541) and streams the weights through pinned host buffers into
 * their device layout.  ctx <= 0 or above the model's context_length means
 * context_length (gpu.go:470-472).  device is the CUDA ordinal. */
LLMB_API int llmb_open(const char *gguf_path, int ctx, int device, llmb_model **out);

/* NewGPU over a reader callback instead of a path; size is the file size. */
LLMB_API int llmb_open_reader(llmb_read_fn read, void *user, uint64_t size, int ctx, int device, llmb_model **out);

/* Releases every device and host resource of the model. */
LLMB_API void llmb_close(llmb_model *m);

/* The message of the last failure on this model; with m == NULL, the last
 * failure of llmb_open / llmb_open_reader on the calling thread.  Never NULL. */
LLMB_API const char *llmb_last_error(const llmb_model *m);

/* GPU.Cfg, gpu.go:119. */
LLMB_API int llmb_get_config(const llmb_model *m, llmb_config *out);

/* GPU.MemoryUsed, gpu.go:766-767: device bytes the model, its cache and its
 * scratch hold. */
LLMB_API uint64_t llmb_memory_used(const llmb_model *m);

/* GPU.Stats, gpu.go:138. */
LLMB_API int llmb_get_stats(const llmb_model *m, llmb_stats *out);

/* Generate, gpu.go:941-1014: greedy decoding.  The prompt goes through the
 * layers in chunks of up to PrefillBatch tokens, then tokens are decoded in
 * launches of DecodeBatch tokens, each sampled on the GPU (first index of the
 * largest logit) from the one before; only the sampled ids come back.
 * Stops after n tokens, at eos (not emitted) or when emit returns 0.  The
 * next launch is queued before the tokens of the one before are read back,
 * so up to 2*DecodeBatch-1 tokens may have been computed past the stop
 * (DecodeBatch-1 in the reference, gpu.go:1048-1051).  Each call starts at
 * position 0.  emit may be NULL.
 * out_tokens (may be NULL) receives the emitted tokens, n_out their count
 * (may be NULL), tm the timing (may be NULL). */
LLMB_API int llmb_generate(llmb_model *m, const int32_t *prompt, int n_prompt, int n, int32_t eos, llmb_emit_fn emit,
                  void *user, int32_t *out_tokens, int *n_out, llmb_timing *tm);

/* Multi-stream generation: n_seq independent greedy sequences on one model
 * (the reference runs one sequence per GPU object; this is the
 * llmb_generate_batch of its multi-stream workload).  Sequence s has the
 * prompt_lens[s] tokens that follow the earlier sequences' in prompts, its
 * own KV cache (the model keeps an arena of n_seq caches), and Generate's
 * semantics (gpu.go:946-1014): at most n tokens, eos stops it and is not
 * emitted.  Each call starts every sequence at position 0.  Prompt tokens
 * of all sequences go through the layers packed PrefillBatch-style in
 * batches of 64; then each step decodes one token of every unfinished
 * sequence, 64 per launch set.  out_tokens receives n_seq rows of n tokens
 * (row s at s * n), n_out (may be NULL) the count of each row, tm (may be
 * NULL) the summed timing. */
LLMB_API int llmb_generate_batch(llmb_model *m, const int32_t *prompts, const int *prompt_lens, int n_seq, int n,
                                 int32_t eos, int32_t *out_tokens, int *n_out, llmb_timing *tm);

/* PrefillLogits, gpu.go:902-927: runs the prompt and copies the vocab
 * logits of its last token into logits (a test hook: Generate never reads
 * logits back). */
LLMB_API int llmb_prefill_logits(llmb_model *m, const int32_t *prompt, int n_prompt, float *logits);

/* A test hook with no single counterpart in the reference: the greedy run
 * of Generate (prompt, then n tokens) that also copies the logits which
 * chose each token into step_logits (n rows of vocab floats), so that a
 * test checks every step against the CPU path, as examples/generate check
 * (main.go:141-181) does for step 1.  Decodes one token per launch. */
LLMB_API int llmb_generate_logits(llmb_model *m, const int32_t *prompt, int n_prompt, int n, int32_t *out_tokens,
                         float *step_logits);

/* Peek, gpu.go:1016-1043: the first n 32-bit words of a named device buffer,
 * as floats.  Names: "x" (residual stream), "q", "att", "gate" (the SwiGLU
 * output), "logits", "state" ({position, step} as raw bits), "tokens",
 * "kvblk.N." (layer N's cache: K then V) and, with the decode_trace knob,
 * "trace" (64-bit globaltimer stamps, see the knob). */
LLMB_API int llmb_peek(llmb_model *m, const char *name, float *out, int n);

/* GPU.Layers, gpu.go:143-146: run only that many layers (debugging: no
 * logits and no sampling are then produced).  0 restores all layers. */
LLMB_API int llmb_set_layers(llmb_model *m, int layers);

/* The package knobs of the reference: "decode_batch" (DecodeBatch,
 * gpu.go:1052, clamped to 1..16 as gpu.go:1046,1054), "prefill_batch"
 * (PrefillBatch, gpu.go:165; read by llmb_open, 1..64) and "memory_budget"
 * (Limits.MemoryBudget, gpu.go:35; bytes, 0 = the device's free memory;
 * read by llmb_open).  One more, with no counterpart in the reference:
 * "decode_mode" 0 (default) decodes with the persistent kernel, 1 with one
 * kernel per phase (an A/B and debugging aid); "prefill_mode" 0 (default)
 * runs prompt chunks and multi-stream batches through the chunked products
 * on the tensor cores (tcgen05, operands split exactly into bf16 pieces,
 * f32 accumulation), 1 through one matvec per token and phase, 2 through
 * chunked products on the FP32 CUDA cores (both A/B aids); "tag_reset" N > 0
 * clears the persistent kernel's tagged exchange buffers after every N
 * decoded tokens (a test aid: they are cleared anyway before the 32-bit tags
 * would wrap); "attn_positions" N (64..256, a multiple of 32; read by
 * llmb_open) sets the positions one attention item of the persistent kernel
 * covers, 0 (default) as many as its shared memory holds (an A/B and test
 * aid: longer contexts are split into items whose partials are merged);
 * "decode_trace" 1 makes models
 * opened afterwards record the persistent kernel's phase timeline, read with
 * llmb_peek(m, "trace", ...) (a profiling aid, the counterpart of GPU.Skip,
 * gpu.go:769-784); "wait_limit_us" N (0 = the default of 2 s) limits
 * every wait of the persistent kernel (a flag poll, a weight slot) to N
 * microseconds, past which the launch stops with LLMB_ERR_DEVICE; and
 * "drop_publish" S >= 0 (-1 = off) makes the persistent kernel skip one
 * publish at decode step S (the step counts prompt tokens too), so that the
 * next phase's wait runs out (a test aid for that error path, with
 * wait_limit_us).  Process-wide, like the Go package variables. */
LLMB_API int llmb_set_knob(const char *name, int64_t value);
LLMB_API int64_t llmb_get_knob(const char *name);

/* Decode attention that allocates no device memory.  It has no counterpart
 * in the reference; it exists for callers that cannot call cudaMalloc: a
 * host whose device memory is a fixed grant made by someone else (the
 * reference runs as a WebAssembly guest whose GPU memory its host grants up
 * front), or code that runs where allocation is not allowed.  Such a caller
 * passes device pointers it already owns:
 *   q        [heads * head_dim]               the query of one position
 *   k_cache  [n_pos rows of kv_stride floats] K, head g at g * head_dim
 *   v_cache  [n_pos rows of kv_stride floats] V, same layout
 *   out      [heads * head_dim]               softmax(q k / sqrt(head_dim)) v
 * (the attention of cpu.go:304-335; query head h reads kv head
 * h / (heads / kv_heads)).  The scratch, split-KV partials, is one
 * fixed array in device memory (about 1 MiB, held by every GPU that loads
 * this library until the process exits), so the sizes are limited: at most
 * 32 heads, head_dim 128 and 4096 positions; larger ones return LLMB_ERR_ARG
 * before any work.  Each call made outside stream capture looks up the
 * array's address on the current device (a host-side query that allocates
 * nothing), so the address always belongs to the current context; a call made
 * while `stream` is capturing a graph reuses the address its device's last
 * call outside capture found, so the first call on a device must come before
 * any capture.  An error already pending on the calling thread
 * (cudaPeekAtLastError) makes the call return LLMB_ERR_CUDA without
 * launching and without clearing it.  Every call shares the array: calls
 * that overlap on the GPU race, so serialise them (one stream).  No part of
 * the array needs clearing between calls: a call reads only what it wrote.
 * Asynchronous on `stream` (a cudaStream_t, NULL for the default stream); the
 * caller synchronises. */
LLMB_API int llmb_attention_noalloc(const float *q, const float *k_cache, const float *v_cache, int n_pos, int heads,
                                    int kv_heads, int head_dim, int kv_stride, float *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LLM_B200_H */
