/*
 * oracle/cpu_ref.c -- the CPU oracle.  TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
 * `--impl reference`) load this library, and only as the checker or as the
 * timed CPU baseline.  The product (llm_b200/libllmb200.so) never links,
 * loads or calls it.
 *
 * What it is: a plain-C restatement of the reference's f32 forward pass,
 * go-wasmcontainers/llm cpu.go (the repository's own equality oracle for its
 * GPU kernels), together with what that file depends on:
 *   - binary16 conversions           f16.go:6-68
 *   - the model configuration        config.go:29-73
 *   - the GGUF v3 header parser      gguf/gguf.go:18-432
 * Every function cites the reference lines it follows.  Go's evaluation order
 * and rounding points are kept: float32 arithmetic rounds after every
 * operation (build with -ffp-contract=off so that no multiply-add is fused,
 * which is what Go does on amd64), and the places where Go goes through
 * float64 (RMSNorm's 1/sqrt, exp in the softmax and SiLU, RoPE's pow and
 * sincos) go through double here too.  Go's own math library is replaced by
 * the C library's exp/pow/sin/cos: both are accurate to about an ulp in
 * double precision, so the float32 results agree except at rare
 * double-rounding boundaries.
 *
 * The reference is Go and no Go toolchain exists here, so it cannot be run to
 * pin this file.  It is pinned instead by the reference's own known-answer
 * tests restated in tests/test_oracle.py (f16 known values, tokenizer_test.go
 * :42-53; the NEOX permutation identity, kernels_test.go:24-58; the GGUF parse
 * and refusal cases, gguf/gguf_test.go:42-78; the 216-file FuzzParse corpus).
 * The forward pass itself has no golden vector that applies to seeded
 * synthetic weights (the reference's testdata JSON files were made by llama.cpp
 * on real instruct weights that are not available), so the forward pass is
 * "parity unpinned" beyond those pieces.
 *
 * Threads: orc_set_threads(n) spreads the rows of each matrix product over n
 * POSIX threads.  Every row is still summed by one thread in the reference's
 * order, so the results are bit-identical for every n.
 */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <pthread.h>

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ f16 -- */

/* F16ToF32, f16.go:6-28: exact conversion, subnormals normalised. */
EXPORT float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1f;
    uint32_t man = (uint32_t)h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            uint32_t e = 127 - 15 + 1;
            while ((man & 0x400) == 0) {
                man <<= 1;
                e--;
            }
            man &= 0x3ff;
            bits = sign | e << 23 | man << 13;
        }
    } else if (exp == 31) {
        bits = sign | 0xffu << 23 | man << 13;
    } else {
        bits = sign | (exp + 127 - 15) << 23 | man << 13;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* F32ToF16, f16.go:30-65: round to nearest even. */
EXPORT uint16_t orc_f32_to_f16(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    uint16_t sign = (uint16_t)(b >> 16) & 0x8000;
    int32_t exp = (int32_t)(b >> 23) & 0xff;
    uint32_t man = b & 0x7fffff;
    if (exp == 0xff) {
        if (man != 0) return sign | 0x7e00;
        return sign | 0x7c00;
    }
    int32_t e = exp - 127 + 15;
    if (e >= 31) return sign | 0x7c00;
    if (e <= 0) {
        if (e < -10) return sign;
        man |= 0x800000;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t h = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1) == 1)) h++;
        return sign | (uint16_t)h;
    }
    uint32_t h = (uint32_t)e << 10 | man >> 13;
    uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1) == 1)) h++;
    return sign | (uint16_t)h;
}

/* RoundF16, f16.go:67-68. */
EXPORT float orc_round_f16(float f) { return orc_f16_to_f32(orc_f32_to_f16(f)); }

/* ----------------------------------------------------------------- GGUF -- */

/* Error classes of gguf/gguf.go:29-34, plus a short read (io.ErrUnexpectedEOF)
 * and the loader's own failures. */
enum {
    ORC_OK = 0,
    ORC_ERR_MAGIC = 1,
    ORC_ERR_VERSION = 2,
    ORC_ERR_BOUND = 3,
    ORC_ERR_FORMAT = 4,
    ORC_ERR_EOF = 5,
    ORC_ERR_CONFIG = 6,
    ORC_ERR_TENSOR = 7,
    ORC_ERR_IO = 8,
    ORC_ERR_CTX = 9,
    ORC_ERR_ARG = 10,
};

/* Bounds, gguf/gguf.go:18-26. */
#define MAX_TENSORS (1ull << 16)
#define MAX_KV (1ull << 16)
#define MAX_STRING (1ull << 24)
#define MAX_ARRAY (1ull << 22)
#define MAX_HEADER (256ull << 20)
#define MAX_DIMS 4
#define MAX_ALIGNMENT (1ull << 20)

/* Metadata value types, gguf/gguf.go:39-54. */
enum { VT_U8, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STRING, VT_ARRAY, VT_U64, VT_I64, VT_F64 };

/* ggml tensor types, gguf/gguf.go:59-69. */
enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q6_K = 14 };

/* Type.BlockSize, gguf/gguf.go:72-92. */
EXPORT int orc_block_size(uint32_t t, uint64_t *elems, uint64_t *bytes) {
    switch (t) {
    case T_F32: *elems = 1, *bytes = 4; return 1;
    case T_F16: *elems = 1, *bytes = 2; return 1;
    case T_Q4_0: *elems = 32, *bytes = 18; return 1;
    case T_Q4_1: *elems = 32, *bytes = 20; return 1;
    case T_Q5_0: *elems = 32, *bytes = 22; return 1;
    case T_Q5_1: *elems = 32, *bytes = 24; return 1;
    case T_Q8_0: *elems = 32, *bytes = 34; return 1;
    case T_Q6_K: *elems = 256, *bytes = 210; return 1;
    }
    *elems = *bytes = 0;
    return 0;
}

/* Go keeps metadata values as uint64, int64, float64, bool, string or []any
 * (gguf/gguf.go:116); the kind says which. */
enum { K_UINT = 1, K_INT, K_FLOAT, K_BOOL, K_STRING, K_ARRAY };

typedef struct {
    char *key;
    int kind;
    uint64_t u;
    int64_t i;
    double f;
    int b;
    char *s;
    uint64_t n; /* array length */
} orc_kv;

typedef struct {
    char *name;
    uint32_t ndims;
    uint64_t dims[MAX_DIMS];
    uint32_t type;
    uint64_t offset, size;
} orc_tensor;

typedef struct orc_gguf {
    uint32_t version;
    orc_kv *kv;
    uint64_t nkv;
    orc_tensor *t;
    uint64_t nt;
    uint64_t data_offset, alignment, size;
} orc_gguf;

/* The bounded reader of gguf/gguf.go:133-208, over bytes in memory: lim is
 * min(size, MaxHeader), and a read past it is ErrBound. */
typedef struct {
    const uint8_t *d;
    uint64_t pos, lim;
} rd_t;

static int rd_read(rd_t *r, void *p, uint64_t n) {
    if (r->pos + n > r->lim) return ORC_ERR_BOUND;
    memcpy(p, r->d + r->pos, n);
    r->pos += n;
    return ORC_OK;
}

static int rd_u32(rd_t *r, uint32_t *v) {
    uint8_t b[4];
    int e = rd_read(r, b, 4);
    if (e) return e;
    *v = (uint32_t)b[0] | (uint32_t)b[1] << 8 | (uint32_t)b[2] << 16 | (uint32_t)b[3] << 24;
    return ORC_OK;
}

static int rd_u64(rd_t *r, uint64_t *v) {
    uint32_t lo, hi;
    int e = rd_u32(r, &lo);
    if (e) return e;
    if ((e = rd_u32(r, &hi))) return e;
    *v = (uint64_t)hi << 32 | lo;
    return ORC_OK;
}

/* reader.str, gguf/gguf.go:195-208. */
static int rd_str(rd_t *r, char **out) {
    uint64_t n;
    int e = rd_u64(r, &n);
    if (e) return e;
    if (n > MAX_STRING) return ORC_ERR_BOUND;
    if (r->pos + n > r->lim) return ORC_ERR_BOUND;
    char *s = malloc(n + 1);
    if (!s) return ORC_ERR_BOUND;
    memcpy(s, r->d + r->pos, n);
    s[n] = 0;
    r->pos += n;
    *out = s;
    return ORC_OK;
}

/* reader.value, gguf/gguf.go:210-289.  Array elements are parsed and
 * checked but only their count is kept (nothing here reads them). */
static int rd_value(rd_t *r, uint32_t t, int depth, orc_kv *kv) {
    uint8_t b[8];
    int e;
    switch (t) {
    case VT_U8: case VT_I8: case VT_BOOL:
        if ((e = rd_read(r, b, 1))) return e;
        if (t == VT_U8) kv->kind = K_UINT, kv->u = b[0];
        else if (t == VT_I8) kv->kind = K_INT, kv->i = (int8_t)b[0];
        else kv->kind = K_BOOL, kv->b = b[0] != 0;
        return ORC_OK;
    case VT_U16: case VT_I16: {
        if ((e = rd_read(r, b, 2))) return e;
        uint16_t v = (uint16_t)(b[0] | b[1] << 8);
        if (t == VT_U16) kv->kind = K_UINT, kv->u = v;
        else kv->kind = K_INT, kv->i = (int16_t)v;
        return ORC_OK;
    }
    case VT_U32: case VT_I32: case VT_F32: {
        uint32_t v;
        if ((e = rd_u32(r, &v))) return e;
        if (t == VT_U32) kv->kind = K_UINT, kv->u = v;
        else if (t == VT_I32) kv->kind = K_INT, kv->i = (int32_t)v;
        else {
            float f;
            memcpy(&f, &v, 4);
            kv->kind = K_FLOAT, kv->f = f;
        }
        return ORC_OK;
    }
    case VT_U64: case VT_I64: case VT_F64: {
        uint64_t v;
        if ((e = rd_u64(r, &v))) return e;
        if (t == VT_U64) kv->kind = K_UINT, kv->u = v;
        else if (t == VT_I64) kv->kind = K_INT, kv->i = (int64_t)v;
        else memcpy(&kv->f, &v, 8), kv->kind = K_FLOAT;
        return ORC_OK;
    }
    case VT_STRING:
        kv->kind = K_STRING;
        return rd_str(r, &kv->s);
    case VT_ARRAY: {
        if (depth > 0) return ORC_ERR_FORMAT; /* nested array */
        uint32_t et;
        uint64_t n;
        if ((e = rd_u32(r, &et))) return e;
        if ((e = rd_u64(r, &n))) return e;
        if (n > MAX_ARRAY) return ORC_ERR_BOUND;
        /* every element takes at least a byte (gguf/gguf.go:273-277) */
        if (n > r->lim - r->pos) return ORC_ERR_BOUND;
        for (uint64_t i = 0; i < n; i++) {
            orc_kv el = {0};
            e = rd_value(r, et, depth + 1, &el);
            free(el.s);
            if (e) return e;
        }
        kv->kind = K_ARRAY, kv->n = n;
        return ORC_OK;
    }
    }
    return ORC_ERR_FORMAT; /* unknown value type */
}

EXPORT void orc_gguf_free(orc_gguf *f) {
    if (!f) return;
    for (uint64_t i = 0; i < f->nkv; i++) free(f->kv[i].key), free(f->kv[i].s);
    for (uint64_t i = 0; i < f->nt; i++) free(f->t[i].name);
    free(f->kv);
    free(f->t);
    free(f);
}

/* Metadata lookup: Go's map keeps the last value written for a key. */
static const orc_kv *gguf_meta(const orc_gguf *f, const char *key) {
    for (uint64_t i = f->nkv; i-- > 0;)
        if (strcmp(f->kv[i].key, key) == 0) return &f->kv[i];
    return NULL;
}

EXPORT int orc_gguf_find(const orc_gguf *f, const char *name) {
    for (uint64_t i = 0; i < f->nt; i++)
        if (strcmp(f->t[i].name, name) == 0) return (int)i;
    return -1;
}

/* Parse, gguf/gguf.go:292-407.  On success *out owns the header. */
EXPORT int orc_gguf_parse(const uint8_t *data, uint64_t size, orc_gguf **out) {
    *out = NULL;
    rd_t r = {data, 0, size < MAX_HEADER ? size : MAX_HEADER};
    uint8_t magic[4];
    int e;
    if ((e = rd_read(&r, magic, 4))) return e;
    if (memcmp(magic, "GGUF", 4) != 0) return ORC_ERR_MAGIC;
    uint32_t ver;
    if ((e = rd_u32(&r, &ver))) return e;
    if (ver != 3) return ORC_ERR_VERSION;
    uint64_t nt, nkv;
    if ((e = rd_u64(&r, &nt))) return e;
    if ((e = rd_u64(&r, &nkv))) return e;
    if (nt > MAX_TENSORS || nkv > MAX_KV) return ORC_ERR_BOUND;
    orc_gguf *f = calloc(1, sizeof *f);
    f->version = ver;
    f->size = size;
    f->kv = calloc(nkv ? nkv : 1, sizeof *f->kv);
    for (uint64_t i = 0; i < nkv; i++) {
        orc_kv *kv = &f->kv[i];
        if ((e = rd_str(&r, &kv->key))) goto fail;
        f->nkv = i + 1;
        uint32_t t;
        if ((e = rd_u32(&r, &t))) goto fail;
        if ((e = rd_value(&r, t, 0, kv))) goto fail;
    }
    f->alignment = 32;
    const orc_kv *a = gguf_meta(f, "general.alignment");
    if (a) {
        if (a->kind != K_UINT || a->u == 0 || a->u > MAX_ALIGNMENT || a->u % 8 != 0) {
            e = ORC_ERR_FORMAT;
            goto fail;
        }
        f->alignment = a->u;
    }
    f->t = calloc(nt ? nt : 1, sizeof *f->t);
    for (uint64_t i = 0; i < nt; i++) {
        orc_tensor *t = &f->t[i];
        if ((e = rd_str(&r, &t->name))) goto fail;
        f->nt = i + 1;
        uint32_t nd;
        if ((e = rd_u32(&r, &nd))) goto fail;
        if (nd == 0 || nd > MAX_DIMS) { e = ORC_ERR_FORMAT; goto fail; }
        t->ndims = nd;
        uint64_t elems = 1;
        for (uint32_t j = 0; j < nd; j++) {
            uint64_t d;
            if ((e = rd_u64(&r, &d))) goto fail;
            if (d == 0 || d > (1ull << 32)) { e = ORC_ERR_BOUND; goto fail; }
            if (elems > (1ull << 62) / d) { e = ORC_ERR_BOUND; goto fail; }
            elems *= d;
            t->dims[j] = d;
        }
        uint32_t ty;
        if ((e = rd_u32(&r, &ty))) goto fail;
        t->type = ty;
        if ((e = rd_u64(&r, &t->offset))) goto fail;
        uint64_t be, bb;
        if (!orc_block_size(ty, &be, &bb)) { e = ORC_ERR_FORMAT; goto fail; }
        if (t->dims[0] % be != 0) { e = ORC_ERR_FORMAT; goto fail; }
        t->size = elems / be * bb;
        for (uint64_t k = 0; k < i; k++)
            if (strcmp(f->t[k].name, t->name) == 0) { e = ORC_ERR_FORMAT; goto fail; }
    }
    f->data_offset = (r.pos + f->alignment - 1) / f->alignment * f->alignment;
    for (uint64_t i = 0; i < f->nt; i++) {
        orc_tensor *t = &f->t[i];
        if (t->offset % f->alignment != 0) { e = ORC_ERR_FORMAT; goto fail; }
        if (t->offset > size || f->data_offset > size - t->offset ||
            t->size > size - f->data_offset - t->offset) {
            e = ORC_ERR_BOUND;
            goto fail;
        }
    }
    *out = f;
    return ORC_OK;
fail:
    orc_gguf_free(f);
    return e;
}

/* File.Uint, gguf/gguf.go:410-420. */
EXPORT int orc_gguf_uint(const orc_gguf *f, const char *key, uint64_t *v) {
    const orc_kv *kv = gguf_meta(f, key);
    *v = 0;
    if (!kv) return 0;
    if (kv->kind == K_UINT) { *v = kv->u; return 1; }
    if (kv->kind == K_INT && kv->i >= 0) { *v = (uint64_t)kv->i; return 1; }
    return 0;
}

/* File.Float, gguf/gguf.go:423-426. */
EXPORT int orc_gguf_float(const orc_gguf *f, const char *key, double *v) {
    const orc_kv *kv = gguf_meta(f, key);
    *v = 0;
    if (!kv || kv->kind != K_FLOAT) return 0;
    *v = kv->f;
    return 1;
}

/* File.Str, gguf/gguf.go:429-432. */
EXPORT const char *orc_gguf_str(const orc_gguf *f, const char *key) {
    const orc_kv *kv = gguf_meta(f, key);
    return kv && kv->kind == K_STRING ? kv->s : NULL;
}

EXPORT uint64_t orc_gguf_ntensors(const orc_gguf *f) { return f->nt; }
EXPORT uint64_t orc_gguf_nkv(const orc_gguf *f) { return f->nkv; }
EXPORT uint64_t orc_gguf_data_offset(const orc_gguf *f) { return f->data_offset; }
EXPORT uint64_t orc_gguf_alignment(const orc_gguf *f) { return f->alignment; }

EXPORT int orc_gguf_tensor(const orc_gguf *f, uint64_t i, const char **name, uint32_t *ndims, uint64_t *dims,
                           uint32_t *type, uint64_t *offset, uint64_t *size) {
    if (i >= f->nt) return ORC_ERR_ARG;
    const orc_tensor *t = &f->t[i];
    *name = t->name;
    *ndims = t->ndims;
    for (uint32_t j = 0; j < MAX_DIMS; j++) dims[j] = j < t->ndims ? t->dims[j] : 0;
    *type = t->type;
    *offset = t->offset;
    *size = t->size;
    return ORC_OK;
}

/* --------------------------------------------------------------- Config -- */

/* Config, config.go:11-23. */
typedef struct {
    int32_t layers, embd, ff, heads, kv_heads, head_dim, vocab, ctx;
    float rope_base, eps;
    int32_t rope_neox, bias, tied_output, arch_qwen2;
} orc_config;

/* ConfigFrom, config.go:29-73.  Returns ORC_ERR_CONFIG with a message. */
static int config_from(const orc_gguf *f, orc_config *c, char *err, int errcap) {
    memset(c, 0, sizeof *c);
    const char *arch = orc_gguf_str(f, "general.architecture");
    if (!arch || (strcmp(arch, "llama") != 0 && strcmp(arch, "qwen2") != 0)) {
        snprintf(err, errcap, "llm: architecture %s is not supported (llama and qwen2 only)", arch ? arch : "\"\"");
        return ORC_ERR_CONFIG;
    }
    char key[256];
#define U(k) (snprintf(key, sizeof key, "%s.%s", arch, k), orc_gguf_uint(f, key, &v), (int64_t)v)
    uint64_t v;
    int64_t layers = U("block_count"), embd = U("embedding_length"), ff = U("feed_forward_length");
    int64_t heads = U("attention.head_count"), kvh = U("attention.head_count_kv"), ctx = U("context_length");
    c->arch_qwen2 = strcmp(arch, "qwen2") == 0;
    c->rope_neox = c->arch_qwen2;
    if (kvh == 0) kvh = heads;
    if (layers <= 0 || embd <= 0 || ff <= 0 || heads <= 0 || kvh <= 0 || embd % heads != 0 || heads % kvh != 0 ||
        layers > INT32_MAX || embd > INT32_MAX || ff > INT32_MAX || ctx > INT32_MAX || ctx < 0) {
        snprintf(err, errcap, "llm: implausible %s hyperparameters", arch);
        return ORC_ERR_CONFIG;
    }
    c->layers = (int32_t)layers, c->embd = (int32_t)embd, c->ff = (int32_t)ff;
    c->heads = (int32_t)heads, c->kv_heads = (int32_t)kvh, c->ctx = (int32_t)ctx;
    c->head_dim = c->embd / c->heads;
    int64_t rd = U("rope.dimension_count");
    if (rd != 0 && rd != c->head_dim) {
        snprintf(err, errcap, "llm: rope.dimension_count %lld differs from the head size %d", (long long)rd, c->head_dim);
        return ORC_ERR_CONFIG;
    }
#undef U
    const char *scal[2] = {"rope.scaling.type", "rope.scaling.factor"};
    for (int i = 0; i < 2; i++) {
        snprintf(key, sizeof key, "%s.%s", arch, scal[i]);
        if (gguf_meta(f, key)) {
            snprintf(err, errcap, "llm: rope scaling (%s) is not supported", key);
            return ORC_ERR_CONFIG;
        }
    }
    double rb, eps;
    snprintf(key, sizeof key, "%s.rope.freq_base", arch);
    if (!orc_gguf_float(f, key, &rb)) rb = 10000;
    snprintf(key, sizeof key, "%s.attention.layer_norm_rms_epsilon", arch);
    orc_gguf_float(f, key, &eps);
    c->rope_base = (float)rb, c->eps = (float)eps;
    int te = orc_gguf_find(f, "token_embd.weight");
    if (te < 0) {
        snprintf(err, errcap, "llm: no token_embd.weight");
        return ORC_ERR_CONFIG;
    }
    /* Go indexes Dims[1] directly (config.go:62); a one-dimensional
     * embedding would panic there, and is an error here. */
    if (f->t[te].ndims < 2 || f->t[te].dims[1] > INT32_MAX) {
        snprintf(err, errcap, "llm: token_embd.weight is not a matrix");
        return ORC_ERR_CONFIG;
    }
    c->vocab = (int32_t)f->t[te].dims[1];
    c->tied_output = orc_gguf_find(f, "output.weight") < 0;
    c->bias = orc_gguf_find(f, "blk.0.attn_q.bias") >= 0;
    if (c->bias != c->arch_qwen2) {
        snprintf(err, errcap, "llm: %s with biases %s is not supported", arch, c->bias ? "true" : "false");
        return ORC_ERR_CONFIG;
    }
    return ORC_OK;
}

/* ---------------------------------------------------------- the kernels -- */

static int g_threads = 1;

EXPORT void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
EXPORT int orc_threads(void) { return g_threads; }

static inline uint16_t u16le(const uint8_t *b) { return (uint16_t)(b[0] | b[1] << 8); }

static inline float f32le(const uint8_t *b) {
    float f;
    memcpy(&f, b, 4);
    return f;
}

/* rmsNorm, cpu.go:81-98 (rmsF64 false): float32 sum of squares in order, then
 * 1/sqrt in float64. */
EXPORT void orc_rmsnorm(float *dst, const float *x, const float *w, int n, float eps) {
    float ss = 0;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float t = ss / (float)n + eps;
    float s = (float)(1.0 / sqrt((double)t));
    for (int i = 0; i < n; i++) dst[i] = x[i] * s * w[i];
}

/* One row of matvec, cpu.go:158-221 (the f32-activation branch, qx == nil). */
static float matvec_row(uint32_t type, int in, const uint8_t *row, const float *x) {
    float sum = 0;
    int nb = in / 32;
    switch (type) {
    case T_Q4_0:
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + (size_t)b * 18;
            float d = orc_f16_to_f32(u16le(blk));
            float s = 0;
            for (int j = 0; j < 16; j++) {
                s += (float)((int)(blk[2 + j] & 15) - 8) * x[b * 32 + j];
                s += (float)((int)(blk[2 + j] >> 4) - 8) * x[b * 32 + j + 16];
            }
            sum += d * s;
        }
        break;
    case T_Q4_1:
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + (size_t)b * 20;
            float d = orc_f16_to_f32(u16le(blk)), mn = orc_f16_to_f32(u16le(blk + 2));
            float s = 0, sx = 0;
            for (int j = 0; j < 16; j++) {
                s += (float)(blk[4 + j] & 15) * x[b * 32 + j];
                s += (float)(blk[4 + j] >> 4) * x[b * 32 + j + 16];
            }
            for (int j = 0; j < 32; j++) sx += x[b * 32 + j];
            sum += d * s + mn * sx;
        }
        break;
    case T_Q8_0:
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + (size_t)b * 34;
            float d = orc_f16_to_f32(u16le(blk));
            float s = 0;
            for (int j = 0; j < 32; j++) s += (float)(int8_t)blk[2 + j] * x[b * 32 + j];
            sum += d * s;
        }
        break;
    }
    return sum;
}

/* A range of rows of one matrix product, for a worker thread. */
typedef struct {
    uint32_t type;
    int in, out;
    size_t row_bytes;
    const uint8_t *data;
    const float *x;
    float *dst;
    int r0, r1;
} mv_job;

static void mv_run(const mv_job *j) {
    for (int o = j->r0; o < j->r1; o++) j->dst[o] = matvec_row(j->type, j->in, j->data + (size_t)j->row_bytes * o, j->x);
}

/* A persistent pool of worker threads: each product hands every worker one
 * contiguous range of rows and waits for all of them. */
static struct {
    pthread_mutex_t mu;
    pthread_cond_t go, done;
    int nworkers;      /* threads started (the caller is worker 0) */
    unsigned long gen; /* job generation */
    int pending;
    mv_job jobs[64];
} pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, PTHREAD_COND_INITIALIZER, 0, 0, 0, {{0}}};

typedef struct {
    int id;
} worker_arg;

static void *pool_worker(void *p) {
    int id = ((worker_arg *)p)->id;
    free(p);
    unsigned long seen = 0;
    for (;;) {
        pthread_mutex_lock(&pool.mu);
        while (pool.gen == seen) pthread_cond_wait(&pool.go, &pool.mu);
        seen = pool.gen;
        mv_job j = pool.jobs[id];
        pthread_mutex_unlock(&pool.mu);
        mv_run(&j);
        pthread_mutex_lock(&pool.mu);
        if (--pool.pending == 0) pthread_cond_signal(&pool.done);
        pthread_mutex_unlock(&pool.mu);
    }
    return NULL;
}

static void pool_matvec(int nt, const mv_job *all) {
    pthread_mutex_lock(&pool.mu);
    while (pool.nworkers < nt - 1) {
        worker_arg *a = malloc(sizeof *a);
        a->id = ++pool.nworkers;
        pthread_t th;
        pthread_create(&th, NULL, pool_worker, a);
        pthread_detach(th);
    }
    for (int i = 1; i < nt; i++) pool.jobs[i] = all[i];
    for (int i = nt; i <= pool.nworkers; i++) pool.jobs[i] = (mv_job){0};
    pool.pending = pool.nworkers;
    pool.gen++;
    pthread_cond_broadcast(&pool.go);
    pthread_mutex_unlock(&pool.mu);
    mv_run(&all[0]);
    pthread_mutex_lock(&pool.mu);
    while (pool.pending > 0) pthread_cond_wait(&pool.done, &pool.mu);
    pthread_mutex_unlock(&pool.mu);
}

/* matvec, cpu.go:142-222: dst = W x for a [in, out] tensor whose rows (ne[0]
 * contiguous) are raw GGUF blocks.  Returns ORC_ERR_TENSOR for a type the
 * reference panics on. */
EXPORT int orc_matvec(uint32_t type, int in, int out, const uint8_t *data, const float *x, float *dst) {
    if (type == T_F32) {
        /* cpu.go:147-157 */
        for (int o = 0; o < out; o++) {
            float s = 0;
            for (int i = 0; i < in; i++) s += f32le(data + 4 * ((size_t)o * in + i)) * x[i];
            dst[o] = s;
        }
        return ORC_OK;
    }
    uint64_t be, bb;
    if (type != T_Q4_0 && type != T_Q4_1 && type != T_Q8_0) return ORC_ERR_TENSOR;
    orc_block_size(type, &be, &bb);
    size_t row_bytes = (size_t)(in / 32) * bb;
    int nt = g_threads;
    if (nt > 64) nt = 64;
    if (nt > out) nt = out;
    if (nt <= 1 || (int64_t)out * in < (1 << 16)) {
        for (int o = 0; o < out; o++) dst[o] = matvec_row(type, in, data + (size_t)o * row_bytes, x);
        return ORC_OK;
    }
    mv_job jobs[64];
    for (int i = 0; i < nt; i++)
        jobs[i] = (mv_job){type, in, out, row_bytes, data, x, dst, (int)((int64_t)out * i / nt), (int)((int64_t)out * (i + 1) / nt)};
    pool_matvec(nt, jobs);
    return ORC_OK;
}

/* rope, cpu.go:368-385: pair i of a head turns by pos * base^(-2i/dim), the
 * angle and its sine and cosine in float64. */
EXPORT void orc_rope(float *x, int pos, int heads, int dim, float base, int neox) {
    for (int h = 0; h < heads; h++) {
        for (int i = 0; i < dim / 2; i++) {
            double theta = (double)pos * pow((double)base, -(double)(2 * i) / (double)dim);
            double s = sin(theta), c = cos(theta);
            int ia = h * dim + 2 * i, ib = h * dim + 2 * i + 1;
            if (neox) ia = h * dim + i, ib = h * dim + i + dim / 2;
            float a = x[ia], b = x[ib];
            x[ia] = a * (float)c - b * (float)s;
            x[ib] = a * (float)s + b * (float)c;
        }
    }
}

/* neoxMap, fused.go:329-334: the row of the NEOX layout that goes to row nr
 * of the adjacent-pair layout, in heads of hd rows. */
EXPORT int orc_neox_map(int nr, int hd) {
    int h = nr / hd, k = nr % hd;
    return h * hd + k / 2 + (k % 2) * (hd / 2);
}

/* Argmax, cpu.go:387-397: the first index of the largest value. */
EXPORT int32_t orc_argmax(const float *l, int n) {
    int best = 0;
    for (int i = 0; i < n; i++)
        if (l[i] > l[best]) best = i;
    return best;
}

/* ---------------------------------------------------------------- model -- */

typedef struct {
    const orc_tensor *t;
    const uint8_t *data;
} tref;

typedef struct {
    tref attn_norm, q, k, v, qb, kb, vb, o, ffn_norm, gate, up, down;
} layer_t;

typedef struct orc_model {
    orc_config c;
    orc_gguf *f;
    uint8_t *map;
    size_t map_len;
    int fd;
    tref emb, out, out_norm;
    layer_t *l;
    float **kc, **vc; /* per layer: ctx * kv_heads * head_dim */
    int pos, max_ctx, max_layers;
    float *last_x;
    /* scratch of Forward, allocated once (cpu.go:230-264 allocates per call) */
    float *x, *h, *q, *kk, *vv, *att, *o, *g, *u, *dn, *scores;
} orc_model;

static int tensor_ref(orc_model *m, const char *name, tref *r, char *err, int errcap) {
    int i = orc_gguf_find(m->f, name);
    if (i < 0) {
        snprintf(err, errcap, "llm: missing tensor %s", name);
        return ORC_ERR_TENSOR;
    }
    r->t = &m->f->t[i];
    r->data = m->map + m->f->data_offset + r->t->offset;
    return ORC_OK;
}

EXPORT void orc_free(orc_model *m) {
    if (!m) return;
    if (m->map) munmap(m->map, m->map_len);
    if (m->fd >= 0) close(m->fd);
    orc_gguf_free(m->f);
    if (m->kc)
        for (int l = 0; l < m->c.layers; l++) free(m->kc[l]), free(m->vc[l]);
    free(m->kc), free(m->vc), free(m->l), free(m->last_x);
    free(m->x), free(m->h), free(m->q), free(m->kk), free(m->vv), free(m->att);
    free(m->o), free(m->g), free(m->u), free(m->dn), free(m->scores);
    free(m);
}

/* LoadCPU, cpu.go:40-61: the file is mapped read-only instead of copied. */
EXPORT int orc_load(const char *path, int max_ctx, orc_model **out, char *err, int errcap) {
    *out = NULL;
    if (errcap > 0) err[0] = 0;
    orc_model *m = calloc(1, sizeof *m);
    m->fd = open(path, O_RDONLY);
    int e = ORC_OK;
    if (m->fd < 0) {
        snprintf(err, errcap, "llm: open %s: %s", path, strerror(errno));
        e = ORC_ERR_IO;
        goto fail;
    }
    struct stat st;
    fstat(m->fd, &st);
    m->map_len = (size_t)st.st_size;
    m->map = mmap(NULL, m->map_len ? m->map_len : 1, PROT_READ, MAP_PRIVATE, m->fd, 0);
    if (m->map == MAP_FAILED) {
        m->map = NULL;
        snprintf(err, errcap, "llm: mmap %s failed", path);
        e = ORC_ERR_IO;
        goto fail;
    }
    if ((e = orc_gguf_parse(m->map, m->map_len, &m->f))) {
        snprintf(err, errcap, "gguf: parse error %d", e);
        goto fail;
    }
    if ((e = config_from(m->f, &m->c, err, errcap))) goto fail;
    orc_config *c = &m->c;
    if (max_ctx <= 0) {
        snprintf(err, errcap, "llm: context of %d", max_ctx);
        e = ORC_ERR_ARG;
        goto fail;
    }
    m->max_ctx = max_ctx;
    if ((e = tensor_ref(m, "token_embd.weight", &m->emb, err, errcap))) goto fail;
    if ((e = tensor_ref(m, "output_norm.weight", &m->out_norm, err, errcap))) goto fail;
    if (c->tied_output) m->out = m->emb;
    else if ((e = tensor_ref(m, "output.weight", &m->out, err, errcap))) goto fail;
    m->l = calloc((size_t)c->layers, sizeof *m->l);
    char name[256];
    for (int l = 0; l < c->layers; l++) {
        layer_t *L = &m->l[l];
#define REF(field, suffix)                                                        \
    snprintf(name, sizeof name, "blk.%d.%s", l, suffix);                          \
    if ((e = tensor_ref(m, name, &L->field, err, errcap))) goto fail;
        REF(attn_norm, "attn_norm.weight")
        REF(q, "attn_q.weight")
        REF(k, "attn_k.weight")
        REF(v, "attn_v.weight")
        REF(o, "attn_output.weight")
        REF(ffn_norm, "ffn_norm.weight")
        REF(gate, "ffn_gate.weight")
        REF(up, "ffn_up.weight")
        REF(down, "ffn_down.weight")
        if (c->bias) {
            REF(qb, "attn_q.bias")
            REF(kb, "attn_k.bias")
            REF(vb, "attn_v.bias")
        }
#undef REF
    }
    size_t kv = (size_t)max_ctx * c->kv_heads * c->head_dim;
    m->kc = calloc((size_t)c->layers, sizeof(float *));
    m->vc = calloc((size_t)c->layers, sizeof(float *));
    for (int l = 0; l < c->layers; l++) {
        m->kc[l] = calloc(kv, sizeof(float));
        m->vc[l] = calloc(kv, sizeof(float));
        if (!m->kc[l] || !m->vc[l]) {
            snprintf(err, errcap, "llm: out of memory for the KV cache");
            e = ORC_ERR_IO;
            goto fail;
        }
    }
    int hd = c->heads * c->head_dim, kvd = c->kv_heads * c->head_dim;
    m->x = calloc(c->embd, 4), m->h = calloc(c->embd, 4), m->q = calloc(hd, 4);
    m->kk = calloc(kvd, 4), m->vv = calloc(kvd, 4), m->att = calloc(hd, 4), m->o = calloc(c->embd, 4);
    m->g = calloc(c->ff, 4), m->u = calloc(c->ff, 4), m->dn = calloc(c->embd, 4);
    m->scores = calloc((size_t)max_ctx, 4), m->last_x = calloc(c->embd, 4);
    *out = m;
    return ORC_OK;
fail:
    orc_free(m);
    return e;
}

EXPORT void orc_get_config(const orc_model *m, orc_config *c) { *c = m->c; }
EXPORT void orc_reset(orc_model *m) { m->pos = 0; }                 /* Reset, cpu.go:63-64 */
EXPORT int orc_pos(const orc_model *m) { return m->pos; }           /* Pos, cpu.go:66-67 */
EXPORT void orc_set_max_layers(orc_model *m, int n) { m->max_layers = n; } /* MaxLayers, cpu.go:29-31 */
EXPORT const float *orc_last_x(const orc_model *m) { return m->last_x; }   /* LastX, cpu.go:32 */

static int mv(const tref *w, const float *x, float *dst) {
    return orc_matvec(w->t->type, (int)w->t->dims[0], (int)w->t->dims[1], w->data, x, dst);
}

/* Forward, cpu.go:224-366 (ExactGGML and F16KV false): one token at the next
 * position.  logits may be NULL; with max_layers set below the layer count
 * no logits are produced (cpu.go:353-356) and 1 is returned.  A full
 * context is an error here where the reference panics (cpu.go:227-229). */
EXPORT int orc_forward(orc_model *m, int32_t tok, float *logits) {
    const orc_config *c = &m->c;
    if (m->pos >= m->max_ctx) return ORC_ERR_CTX;
    if (tok < 0 || tok >= c->vocab) return ORC_ERR_ARG;
    float *x = m->x, *h = m->h, *q = m->q, *kk = m->kk, *vv = m->vv, *att = m->att;
    float *o = m->o, *g = m->g, *u = m->u, *dn = m->dn, *scores = m->scores;
    /* embedding row, cpu.go:231-254 */
    switch (m->emb.t->type) {
    case T_Q8_0: {
        size_t rb = (size_t)c->embd / 32 * 34;
        const uint8_t *row = m->emb.data + (size_t)tok * rb;
        for (int b = 0; b < c->embd / 32; b++) {
            float d = orc_f16_to_f32(u16le(row + b * 34));
            for (int j = 0; j < 32; j++) x[b * 32 + j] = d * (float)(int8_t)row[b * 34 + 2 + j];
        }
        break;
    }
    case T_Q4_0: {
        size_t rb = (size_t)c->embd / 32 * 18;
        const uint8_t *row = m->emb.data + (size_t)tok * rb;
        for (int b = 0; b < c->embd / 32; b++) {
            float d = orc_f16_to_f32(u16le(row + b * 18));
            for (int j = 0; j < 16; j++) {
                x[b * 32 + j] = d * (float)((int)(row[b * 18 + 2 + j] & 15) - 8);
                x[b * 32 + j + 16] = d * (float)((int)(row[b * 18 + 2 + j] >> 4) - 8);
            }
        }
        break;
    }
    default:
        return ORC_ERR_TENSOR;
    }
    int kvd = c->kv_heads * c->head_dim;
    int nl = c->layers;
    if (m->max_layers != 0) {
        int ml = m->max_layers > 0 ? m->max_layers : 0;
        nl = nl < ml ? nl : ml;
    }
    int e;
    for (int l = 0; l < nl; l++) {
        const layer_t *L = &m->l[l];
        orc_rmsnorm(h, x, (const float *)L->attn_norm.data, c->embd, c->eps); /* cpu.go:279 */
        if ((e = mv(&L->q, h, q)) || (e = mv(&L->k, h, kk)) || (e = mv(&L->v, h, vv))) return e;
        if (c->bias) { /* cpu.go:284-294 */
            for (int i = 0; i < (int)L->qb.t->dims[0]; i++) q[i] += f32le(L->qb.data + 4 * i);
            for (int i = 0; i < (int)L->kb.t->dims[0]; i++) kk[i] += f32le(L->kb.data + 4 * i);
            for (int i = 0; i < (int)L->vb.t->dims[0]; i++) vv[i] += f32le(L->vb.data + 4 * i);
        }
        orc_rope(q, m->pos, c->heads, c->head_dim, c->rope_base, c->rope_neox); /* cpu.go:295-296 */
        orc_rope(kk, m->pos, c->kv_heads, c->head_dim, c->rope_base, c->rope_neox);
        for (int i = 0; i < kvd; i++) { /* cpu.go:297-303 */
            m->kc[l][(size_t)m->pos * kvd + i] = kk[i];
            m->vc[l][(size_t)m->pos * kvd + i] = vv[i];
        }
        float scale = (float)(1.0 / sqrt((double)c->head_dim)); /* cpu.go:304 */
        int grp = c->heads / c->kv_heads;
        for (int hd = 0; hd < c->heads; hd++) { /* cpu.go:306-335 */
            int kvh = hd / grp;
            const float *qv = q + hd * c->head_dim;
            float mx = -INFINITY;
            for (int t = 0; t <= m->pos; t++) {
                const float *kr = m->kc[l] + (size_t)t * kvd + kvh * c->head_dim;
                float s = 0;
                for (int i = 0; i < c->head_dim; i++) s += qv[i] * kr[i];
                scores[t] = s * scale;
                mx = scores[t] > mx ? scores[t] : mx;
            }
            float sum = 0;
            for (int t = 0; t <= m->pos; t++) {
                scores[t] = (float)exp((double)(scores[t] - mx));
                sum += scores[t];
            }
            float *outv = att + hd * c->head_dim;
            for (int i = 0; i < c->head_dim; i++) outv[i] = 0;
            for (int t = 0; t <= m->pos; t++) {
                const float *vr = m->vc[l] + (size_t)t * kvd + kvh * c->head_dim;
                float w = scores[t] / sum;
                for (int i = 0; i < c->head_dim; i++) outv[i] += w * vr[i];
            }
        }
        if ((e = mv(&L->o, att, o))) return e; /* cpu.go:336-339 */
        for (int i = 0; i < c->embd; i++) x[i] += o[i];
        orc_rmsnorm(h, x, (const float *)L->ffn_norm.data, c->embd, c->eps); /* cpu.go:340 */
        if ((e = mv(&L->gate, h, g)) || (e = mv(&L->up, h, u))) return e;
        for (int i = 0; i < c->ff; i++) g[i] = g[i] / (1 + (float)exp((double)-g[i])) * u[i]; /* cpu.go:344-346 */
        if ((e = mv(&L->down, g, dn))) return e; /* cpu.go:347-350 */
        for (int i = 0; i < c->embd; i++) x[i] += dn[i];
    }
    memcpy(m->last_x, x, (size_t)c->embd * 4); /* cpu.go:352 */
    if (m->max_layers != 0 && m->max_layers < c->layers) {
        m->pos++;
        return 1;
    }
    orc_rmsnorm(h, x, (const float *)m->out_norm.data, c->embd, c->eps); /* cpu.go:357-363 */
    if (logits) {
        if ((e = mv(&m->out, h, logits))) return e;
    } else {
        float *tmp = malloc((size_t)c->vocab * 4);
        e = mv(&m->out, h, tmp);
        free(tmp);
        if (e) return e;
    }
    m->pos++;
    return ORC_OK;
}

/* The greedy loop the reference's tests and `check` drive (oracle_test.go
 * :139-152, examples/generate/main.go:154-175): reset, the prompt through
 * Forward, then n tokens, each the argmax of the logits before it.
 * step_logits, if not NULL, receives n rows of vocab floats: row 0 the
 * logits after the prompt (which gave token 0), row i those that gave token
 * i.  Stops early (returning ORC_ERR_CTX) when the context is full. */
EXPORT int orc_generate(orc_model *m, const int32_t *prompt, int n_prompt, int n, int32_t *tokens, float *step_logits) {
    const orc_config *c = &m->c;
    if (n_prompt <= 0) return ORC_ERR_ARG;
    float *logits = malloc((size_t)c->vocab * 4);
    int e = ORC_OK;
    orc_reset(m);
    for (int i = 0; i < n_prompt && !e; i++) e = orc_forward(m, prompt[i], logits);
    for (int i = 0; i < n && !e; i++) {
        if (step_logits) memcpy(step_logits + (size_t)i * c->vocab, logits, (size_t)c->vocab * 4);
        tokens[i] = orc_argmax(logits, c->vocab);
        if (i + 1 < n) e = orc_forward(m, tokens[i], logits);
    }
    free(logits);
    return e;
}
