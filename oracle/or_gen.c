/* Oracle generators: the reference's fixture models (tests/TinyModels.cs, tests/TinyMoe.cs) restated byte for byte,
 * a GGUF writer (GgufWriter, tests/TinyModels.cs:11-86), round-to-nearest block quantizers and the counter-based
 * synthetic weights the CUDA generator reproduces bit for bit. Test infrastructure only (see oracle.h). */
#include "oracle.h"
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---------------- xorshift64* (tests/TinyModels.cs:89-97) ---------------- */
void or_rng_init(or_rng* r, uint64_t seed) { r->s = seed * 0x9E3779B97F4A7C15ULL + 1; }
uint64_t or_rng_next(or_rng* r) { r->s ^= r->s >> 12; r->s ^= r->s << 25; r->s ^= r->s >> 27; return r->s * 2685821657736338717ULL; }
uint8_t or_rng_byte(or_rng* r) { return (uint8_t)(or_rng_next(r) >> 56); }
double or_rng_uniform(or_rng* r) { return (double)(or_rng_next(r) >> 11) * (1.0 / 9007199254740992.0); }
float or_rng_normal(or_rng* r)
{
    double u = or_rng_uniform(r); if (u < 1e-12) u = 1e-12;
    double v = or_rng_uniform(r);
    return (float)(sqrt(-2 * log(u)) * cos(2 * M_PI * v));
}

/* ---------------- GgufWriter (tests/TinyModels.cs:11-86) ---------------- */
typedef struct { char* key; int type; int arr_type; void* data; int64_t n; } wkv;   /* type: 8 str, 4 u32, 5 i32, 6 f32, 7 bool, 9 array */
typedef struct { char* name; int64_t dims[4]; int nd; int type; uint8_t* data; int64_t len; } wten;
typedef struct { wkv* kv; int nkv, ckv; wten* t; int nt, ct; } gw;

static void gw_add(gw* w, const char* key, int type, int arr_type, const void* data, int64_t n, size_t elem)
{
    if (w->nkv == w->ckv) { w->ckv = w->ckv ? 2 * w->ckv : 32; w->kv = (wkv*)realloc(w->kv, sizeof(wkv) * (size_t)w->ckv); }
    wkv* k = &w->kv[w->nkv++];
    k->key = strdup(key); k->type = type; k->arr_type = arr_type; k->n = n;
    if (type == 8) k->data = strdup((const char*)data);
    else if (type == 9 && arr_type == 8) {
        char** src = (char**)data; char** dst = (char**)malloc(sizeof(char*) * (size_t)n);
        for (int64_t i = 0; i < n; i++) dst[i] = strdup(src[i]);
        k->data = dst;
    } else { k->data = malloc(elem * (size_t)(n > 0 ? n : 1)); memcpy(k->data, data, elem * (size_t)n); }
}
static void gw_str(gw* w, const char* key, const char* v) { gw_add(w, key, 8, 0, v, 1, 0); }
static void gw_u32(gw* w, const char* key, uint32_t v) { gw_add(w, key, 4, 0, &v, 1, 4); }
static void gw_f32(gw* w, const char* key, float v) { gw_add(w, key, 6, 0, &v, 1, 4); }
static void gw_bool(gw* w, const char* key, int v) { uint8_t b = v ? 1 : 0; gw_add(w, key, 7, 0, &b, 1, 1); }
static void gw_strs(gw* w, const char* key, char** v, int n) { gw_add(w, key, 9, 8, v, n, 0); }
static void gw_i32s(gw* w, const char* key, const int32_t* v, int n) { gw_add(w, key, 9, 5, v, n, 4); }
static void gw_f32s(gw* w, const char* key, const float* v, int n) { gw_add(w, key, 9, 6, v, n, 4); }

static void gw_tensor(gw* w, const char* name, int type, uint8_t* data, int64_t len, int nd, int64_t d0, int64_t d1, int64_t d2)
{
    if (w->nt == w->ct) { w->ct = w->ct ? 2 * w->ct : 64; w->t = (wten*)realloc(w->t, sizeof(wten) * (size_t)w->ct); }
    wten* t = &w->t[w->nt++];
    t->name = strdup(name); t->type = type; t->data = data; t->len = len; t->nd = nd;
    t->dims[0] = d0; t->dims[1] = d1; t->dims[2] = d2; t->dims[3] = 1;
}

static void put_str(FILE* f, const char* s) { uint64_t n = strlen(s); fwrite(&n, 8, 1, f); fwrite(s, 1, n, f); }
static void pad32(FILE* f) { long p = ftell(f); static const uint8_t z[32] = {0}; if (p % 32) fwrite(z, 1, (size_t)(32 - p % 32), f); }

static int gw_save(gw* w, const char* path)
{
    FILE* f = fopen(path, "wb");
    if (!f) return -1;
    uint32_t magic = 0x46554747u, version = 3;
    int64_t nt = w->nt, nkv = w->nkv;
    fwrite(&magic, 4, 1, f); fwrite(&version, 4, 1, f); fwrite(&nt, 8, 1, f); fwrite(&nkv, 8, 1, f);
    for (int i = 0; i < w->nkv; i++) {
        wkv* k = &w->kv[i];
        put_str(f, k->key);
        int32_t ty = k->type; fwrite(&ty, 4, 1, f);
        if (k->type == 8) put_str(f, (const char*)k->data);
        else if (k->type == 9) {
            int32_t at = k->arr_type; fwrite(&at, 4, 1, f); fwrite(&k->n, 8, 1, f);
            if (k->arr_type == 8) for (int64_t j = 0; j < k->n; j++) put_str(f, ((char**)k->data)[j]);
            else fwrite(k->data, 4, (size_t)k->n, f);
        } else if (k->type == 7) fwrite(k->data, 1, 1, f);
        else fwrite(k->data, 4, 1, f);
    }
    uint64_t off = 0;
    for (int i = 0; i < w->nt; i++) {
        wten* t = &w->t[i];
        put_str(f, t->name);
        uint32_t nd = (uint32_t)t->nd; fwrite(&nd, 4, 1, f);
        for (int d = 0; d < t->nd; d++) fwrite(&t->dims[d], 8, 1, f);
        int32_t ty = t->type; fwrite(&ty, 4, 1, f);
        fwrite(&off, 8, 1, f);
        off += (uint64_t)((t->len + 31) / 32 * 32);
    }
    pad32(f);
    for (int i = 0; i < w->nt; i++) { fwrite(w->t[i].data, 1, (size_t)w->t[i].len, f); pad32(f); }
    int bad = ferror(f);
    fclose(f);
    return bad ? -1 : 0;
}

static void gw_free(gw* w)
{
    for (int i = 0; i < w->nkv; i++) {
        wkv* k = &w->kv[i];
        if (k->type == 9 && k->arr_type == 8) for (int64_t j = 0; j < k->n; j++) free(((char**)k->data)[j]);
        free(k->data); free(k->key);
    }
    for (int i = 0; i < w->nt; i++) { free(w->t[i].name); free(w->t[i].data); }
    free(w->kv); free(w->t);
}

/* ---------------- vocabularies (tests/TinyModels.cs:117-169) ---------------- */
static const char* BPE_MERGES[40] = {
    "\xc4\xa0 t", "h e", "\xc4\xa0t he", "i n", "\xc4\xa0 a", "e r", "o n", "\xc4\xa0 w", "r e", "\xc4\xa0 s", "a t", "o r", "e n", "\xc4\xa0 o", "\xc4\xa0 c",
    "i s", "a n", "\xc4\xa0 b", "l l", "\xc4\xa0 h", "e s", "i t", "\xc4\xa0 l", "\xc4\xa0 d", "\xc4\xa0 in", "\xc4\xa0 f", "a r", "\xc4\xa0 m", "\xc4\xa0 p", "o u",
    "\xc4\xa0w or", "l d", "\xc4\xa0wor ld", "\xc4\xa0 is", "H e", "He ll", "Hell o", "\xc4\xa0 1", "\xc4\xa0 2", "\xc4\x8a \xc4\x8a"
};
static const char* SPM_PIECES[23] = {
    "\xe2\x96\x81", "\xe2\x96\x81t", "he", "\xe2\x96\x81the", "\xe2\x96\x81""a", "er", "on", "\xe2\x96\x81w", "re", "\xe2\x96\x81s", "in",
    "\xe2\x96\x81the\xe2\x96\x81", "\xe2\x96\x81world", "\xe2\x96\x81is", "\xe2\x96\x81Hello", "ll", "\xe2\x96\x81H", "\xe2\x96\x81[", "INST", "]", "[/",
    "\xe2\x96\x81[/INST]", "\xe2\x96\x81[INST]"
};

static void utf8(unsigned cp, char* out)
{
    if (cp < 0x80) { out[0] = (char)cp; out[1] = 0; }
    else if (cp < 0x800) { out[0] = (char)(0xC0 | (cp >> 6)); out[1] = (char)(0x80 | (cp & 0x3F)); out[2] = 0; }
    else { out[0] = (char)(0xE0 | (cp >> 12)); out[1] = (char)(0x80 | ((cp >> 6) & 0x3F)); out[2] = (char)(0x80 | (cp & 0x3F)); out[3] = 0; }
}

/* ByteChar (tests/TinyModels.cs:140-150): GPT-2's byte-to-unicode map. */
static unsigned byte_char(int b)
{
    int n = 0;
    for (int i = 0; i < 256; i++) {
        int printable = (i >= 0x21 && i <= 0x7E) || (i >= 0xA1 && i <= 0xAC) || (i >= 0xAE && i <= 0xFF);
        unsigned c = printable ? (unsigned)i : (unsigned)(256 + n++);
        if (i == b) return c;
    }
    return 0;
}

typedef struct { char** tok; int32_t* type; float* score; int n; char** merges; int nmerges; int bos, eos; } vocab_t;

static void vocab_free(vocab_t* v)
{
    for (int i = 0; i < v->n; i++) free(v->tok[i]);
    for (int i = 0; i < v->nmerges; i++) free(v->merges[i]);
    free(v->tok); free(v->type); free(v->score); free(v->merges);
}

static char* strip_spaces(const char* s)
{
    char* o = (char*)malloc(strlen(s) + 1); int k = 0;
    for (; *s; s++) if (*s != ' ') o[k++] = *s;
    o[k] = 0; return o;
}

static void bpe_vocab(int llama, vocab_t* v)
{
    memset(v, 0, sizeof(*v));
    int cap = 256 + 40 + 5;
    v->tok = (char**)calloc((size_t)cap, sizeof(char*)); v->type = (int32_t*)calloc((size_t)cap, 4);
    char buf[8];
    for (int b = 0; b < 256; b++) { utf8(byte_char(b), buf); v->tok[v->n] = strdup(buf); v->type[v->n++] = 1; }
    for (int i = 0; i < 40; i++) { v->tok[v->n] = strip_spaces(BPE_MERGES[i]); v->type[v->n++] = 1; }
    const char* sl[] = { "<|begin_of_text|>", "<|end_of_text|>", "<|start_header_id|>", "<|end_header_id|>", "<|eot_id|>" };
    const char* sq[] = { "<|endoftext|>", "<|im_start|>", "<|im_end|>" };
    int ns = llama ? 5 : 3;
    for (int i = 0; i < ns; i++) { v->tok[v->n] = strdup(llama ? sl[i] : sq[i]); v->type[v->n++] = 3; }
    v->merges = (char**)calloc(40, sizeof(char*)); v->nmerges = 40;
    for (int i = 0; i < 40; i++) v->merges[i] = strdup(BPE_MERGES[i]);
    v->bos = llama ? 296 : 296;       /* index of <|begin_of_text|> / <|endoftext|> */
    v->eos = llama ? 300 : 298;       /* index of <|eot_id|> / <|im_end|> */
}

static void spm_vocab(vocab_t* v)
{
    memset(v, 0, sizeof(*v));
    int cap = 3 + 256 + 26 + 26 + 23;
    v->tok = (char**)calloc((size_t)cap, sizeof(char*)); v->type = (int32_t*)calloc((size_t)cap, 4); v->score = (float*)calloc((size_t)cap, 4);
    const char* first[] = { "<unk>", "<s>", "</s>" }; int ft[] = { 2, 3, 3 };
    for (int i = 0; i < 3; i++) { v->tok[v->n] = strdup(first[i]); v->type[v->n] = ft[i]; v->score[v->n++] = 0; }
    char buf[16];
    for (int b = 0; b < 256; b++) { snprintf(buf, sizeof buf, "<0x%02X>", b); v->tok[v->n] = strdup(buf); v->type[v->n] = 6; v->score[v->n++] = 0; }
    for (char c = 'a'; c <= 'z'; c++) { buf[0] = c; buf[1] = 0; v->tok[v->n] = strdup(buf); v->type[v->n] = 1; v->score[v->n++] = (float)(-100 - (c - 'a')); }
    for (char c = 'A'; c <= 'Z'; c++) { buf[0] = c; buf[1] = 0; v->tok[v->n] = strdup(buf); v->type[v->n] = 1; v->score[v->n++] = (float)(-200 - (c - 'A')); }
    for (int i = 0; i < 23; i++) { v->tok[v->n] = strdup(SPM_PIECES[i]); v->type[v->n] = 1; v->score[v->n++] = -i * 1.5f; }
    v->bos = 1; v->eos = 2;
}

/* ---------------- TinyModels.Matrix (tests/TinyModels.cs:314-381) ---------------- */
static int scale_fields(int t, int* f)
{
    switch (t) {
    case OR_Q4_0: case OR_Q5_0: case OR_Q8_0: f[0] = 0; return 1;
    case OR_Q4_1: case OR_Q5_1: case OR_Q4_K: case OR_Q5_K: f[0] = 0; f[1] = 2; return 2;
    case OR_Q2_K: f[0] = 80; f[1] = 82; return 2;
    case OR_Q3_K: f[0] = 108; return 1;
    case OR_Q6_K: f[0] = 208; return 1;
    case OR_IQ4_NL: case OR_IQ4_XS: case OR_IQ3_XXS: case OR_IQ3_S: case OR_IQ2_XXS: case OR_IQ2_XS: case OR_IQ2_S: case OR_IQ1_S: f[0] = 0; return 1;
    case OR_IQ1_M: return 0;
    }
    return -1;
}

static void put_scale(uint8_t* data, int64_t o, int t, const int* fields, int nf, uint16_t h)
{
    if (t == OR_IQ1_M) {
        for (int k = 0; k < 4; k++) data[o + 48 + 2 * k + 1] = (uint8_t)((data[o + 48 + 2 * k + 1] & 0x0F) | (((h >> (4 * k)) & 0xF) << 4));
        return;
    }
    for (int i = 0; i < nf; i++) { data[o + fields[i]] = (uint8_t)h; data[o + fields[i] + 1] = (uint8_t)(h >> 8); }
}

int or_matrix(or_rng* rng, int t, int rows, int cols, float rms, uint8_t* data)
{
    int bs, ts;
    if (!or_layout(t, &bs, &ts)) return -1;
    int64_t n = (int64_t)rows * cols, len = n / bs * ts;
    if (t == OR_F32 || t == OR_F16 || t == OR_BF16) {
        for (int64_t i = 0; i < n; i++) {
            float v = rms * or_rng_normal(rng);
            if (t == OR_F32) memcpy(data + i * 4, &v, 4);
            else {
                uint32_t bits; memcpy(&bits, &v, 4);
                uint16_t h = t == OR_F16 ? or_float_to_half(v) : (uint16_t)(bits >> 16);
                data[i * 2] = (uint8_t)h; data[i * 2 + 1] = (uint8_t)(h >> 8);
            }
        }
        return 0;
    }
    for (int64_t i = 0; i < len; i++) data[i] = or_rng_byte(rng);
    int fields[2]; int nf = scale_fields(t, fields);
    if (nf < 0) return -1;
    int64_t blocks = len / ts;
    float* tmp = (float*)malloc(sizeof(float) * (size_t)bs);
    for (int64_t b = 0; b < blocks; b++) {
        int64_t o = b * ts;
        put_scale(data, o, t, fields, nf, or_float_to_half(1.0f));
        double sum = 0;
        or_decode_row(t, data + o, bs, tmp);
        for (int i = 0; i < bs; i++) { float v = tmp[i]; sum += (double)(v * v); }
        double ms = sum / bs; if (ms < 1e-12) ms = 1e-12;
        float scale = (float)((double)rms / sqrt(ms));
        scale *= (float)(0.75 + 0.5 * or_rng_uniform(rng));
        put_scale(data, o, t, fields, nf, or_float_to_half(scale));
    }
    free(tmp);
    return 0;
}

static uint8_t* mat(or_rng* rng, int t, int rows, int cols, float rms, int64_t* len)
{
    int bs, ts; or_layout(t, &bs, &ts);
    *len = (int64_t)rows * cols / bs * ts;
    uint8_t* d = (uint8_t*)malloc((size_t)*len);
    or_matrix(rng, t, rows, cols, rms, d);
    return d;
}
static uint8_t* f32v(const float* v, int n, int64_t* len) { *len = (int64_t)n * 4; uint8_t* d = (uint8_t*)malloc((size_t)*len); memcpy(d, v, (size_t)*len); return d; }
static uint8_t* normv(or_rng* rng, int n, int64_t* len)
{
    float* v = (float*)malloc(sizeof(float) * (size_t)n);
    for (int i = 0; i < n; i++) v[i] = 1.0f + 0.2f * or_rng_normal(rng);
    uint8_t* d = f32v(v, n, len); free(v); return d;
}
static uint8_t* vecv(or_rng* rng, int n, float scale, int64_t* len)
{
    float* v = (float*)malloc(sizeof(float) * (size_t)n);
    for (int i = 0; i < n; i++) v[i] = scale * or_rng_normal(rng);
    uint8_t* d = f32v(v, n, len); free(v); return d;
}

static const char* type_name(int t)
{
    switch (t) {
    case OR_F32: return "f32"; case OR_F16: return "f16"; case OR_BF16: return "bf16"; case OR_Q4_0: return "q4_0";
    case OR_Q4_1: return "q4_1"; case OR_Q5_0: return "q5_0"; case OR_Q5_1: return "q5_1"; case OR_Q8_0: return "q8_0";
    case OR_Q2_K: return "q2_K"; case OR_Q3_K: return "q3_K"; case OR_Q4_K: return "q4_K"; case OR_Q5_K: return "q5_K";
    case OR_Q6_K: return "q6_K"; case OR_IQ2_XXS: return "iq2_xxs"; case OR_IQ2_XS: return "iq2_xs"; case OR_IQ3_XXS: return "iq3_xxs";
    case OR_IQ1_S: return "iq1_s"; case OR_IQ4_NL: return "iq4_nl"; case OR_IQ3_S: return "iq3_s"; case OR_IQ2_S: return "iq2_s";
    case OR_IQ4_XS: return "iq4_xs"; case OR_IQ1_M: return "iq1_m";
    }
    return "unknown";
}

static void add_bpe_meta(gw* w, int llama, int* vocab_out)
{
    vocab_t v; bpe_vocab(llama, &v);
    gw_str(w, "tokenizer.ggml.model", "gpt2");
    gw_str(w, "tokenizer.ggml.pre", llama ? "llama-bpe" : "qwen2");
    gw_strs(w, "tokenizer.ggml.tokens", v.tok, v.n);
    gw_i32s(w, "tokenizer.ggml.token_type", v.type, v.n);
    gw_strs(w, "tokenizer.ggml.merges", v.merges, v.nmerges);
    gw_u32(w, "tokenizer.ggml.bos_token_id", (uint32_t)(llama ? 296 : 296));
    gw_u32(w, "tokenizer.ggml.eos_token_id", (uint32_t)(llama ? 300 : 298));
    gw_bool(w, "tokenizer.ggml.add_bos_token", llama);
    gw_str(w, "tokenizer.chat_template", llama ? "{{ '<|start_header_id|>' }}" : "{{ '<|im_start|>' }}");
    *vocab_out = v.n;
    vocab_free(&v);
}

/* TinyModels.Build (tests/TinyModels.cs:204-291). */
int or_write_tiny(const char* path, const char* arch, int type, int flags, int layers, int embd, int heads,
                  int kv_heads, int ff, uint64_t seed)
{
    int tied = flags & 1, spm = flags & 2, rope_freqs = flags & 4;
    int is_llama = strcmp(arch, "llama") == 0, is_qwen2 = strcmp(arch, "qwen2") == 0, is_qwen3 = strcmp(arch, "qwen3") == 0;
    or_rng rng; or_rng_init(&rng, seed);
    gw w; memset(&w, 0, sizeof w);
    char a[64], key[128], name[128];
    snprintf(a, sizeof a, "%s.", arch);
    int hd = embd / heads;
    gw_str(&w, "general.architecture", arch);
    snprintf(name, sizeof name, "tiny-%s-%s%s%s%s", arch, type_name(type), tied ? "-tied" : "", spm ? "-spm" : "", rope_freqs ? "-ropefreqs" : "");
    gw_str(&w, "general.name", name);
    gw_u32(&w, "general.alignment", 32);
#define K(s) (snprintf(key, sizeof key, "%s%s", a, s), key)
    gw_u32(&w, K("block_count"), (uint32_t)layers);
    gw_u32(&w, K("context_length"), 512);
    gw_u32(&w, K("embedding_length"), (uint32_t)embd);
    gw_u32(&w, K("feed_forward_length"), (uint32_t)ff);
    gw_u32(&w, K("attention.head_count"), (uint32_t)heads);
    gw_u32(&w, K("attention.head_count_kv"), (uint32_t)kv_heads);
    gw_f32(&w, K("attention.layer_norm_rms_epsilon"), 1e-5f);
    gw_f32(&w, K("rope.freq_base"), is_llama ? 500000.0f : 1000000.0f);
    if (is_qwen3) { gw_u32(&w, K("attention.key_length"), (uint32_t)hd); gw_u32(&w, K("attention.value_length"), (uint32_t)hd); }
    if (is_llama) gw_u32(&w, K("rope.dimension_count"), (uint32_t)hd);
    int vocab;
    if (spm) {
        vocab_t v; spm_vocab(&v);
        gw_str(&w, "tokenizer.ggml.model", "llama");
        gw_strs(&w, "tokenizer.ggml.tokens", v.tok, v.n);
        gw_f32s(&w, "tokenizer.ggml.scores", v.score, v.n);
        gw_i32s(&w, "tokenizer.ggml.token_type", v.type, v.n);
        gw_u32(&w, "tokenizer.ggml.bos_token_id", 1);
        gw_u32(&w, "tokenizer.ggml.eos_token_id", 2);
        gw_u32(&w, "tokenizer.ggml.unknown_token_id", 0);
        gw_str(&w, "tokenizer.chat_template", "{{ bos_token }}{% for message in messages %}[INST] {{ message['content'] }} [/INST]{% endfor %}");
        vocab = v.n; vocab_free(&v);
    } else add_bpe_meta(&w, is_llama, &vocab);

    int qd = heads * hd, kd = kv_heads * hd;
    int64_t len; uint8_t* d;
    d = mat(&rng, type, vocab, embd, 1.0f, &len); gw_tensor(&w, "token_embd.weight", type, d, len, 2, embd, vocab, 1);
    if (rope_freqs) {
        float* f = (float*)malloc(sizeof(float) * (size_t)(hd / 2));
        for (int i = 0; i < hd / 2; i++) f[i] = 1.0f + i * 0.25f;
        d = f32v(f, hd / 2, &len); free(f);
        gw_tensor(&w, "rope_freqs.weight", OR_F32, d, len, 1, hd / 2, 1, 1);
    }
    for (int l = 0; l < layers; l++) {
        char p[32]; snprintf(p, sizeof p, "blk.%d.", l);
#define N(s) (snprintf(name, sizeof name, "%s%s", p, s), name)
        d = normv(&rng, embd, &len); gw_tensor(&w, N("attn_norm.weight"), OR_F32, d, len, 1, embd, 1, 1);
        d = mat(&rng, type, qd, embd, 0.08f, &len); gw_tensor(&w, N("attn_q.weight"), type, d, len, 2, embd, qd, 1);
        d = mat(&rng, type, kd, embd, 0.08f, &len); gw_tensor(&w, N("attn_k.weight"), type, d, len, 2, embd, kd, 1);
        d = mat(&rng, type, kd, embd, 0.08f, &len); gw_tensor(&w, N("attn_v.weight"), type, d, len, 2, embd, kd, 1);
        if (is_qwen2) {
            d = vecv(&rng, qd, 0.1f, &len); gw_tensor(&w, N("attn_q.bias"), OR_F32, d, len, 1, qd, 1, 1);
            d = vecv(&rng, kd, 0.1f, &len); gw_tensor(&w, N("attn_k.bias"), OR_F32, d, len, 1, kd, 1, 1);
            d = vecv(&rng, kd, 0.1f, &len); gw_tensor(&w, N("attn_v.bias"), OR_F32, d, len, 1, kd, 1, 1);
        }
        if (is_qwen3) {
            d = normv(&rng, hd, &len); gw_tensor(&w, N("attn_q_norm.weight"), OR_F32, d, len, 1, hd, 1, 1);
            d = normv(&rng, hd, &len); gw_tensor(&w, N("attn_k_norm.weight"), OR_F32, d, len, 1, hd, 1, 1);
        }
        d = mat(&rng, type, embd, qd, 0.08f, &len); gw_tensor(&w, N("attn_output.weight"), type, d, len, 2, qd, embd, 1);
        d = normv(&rng, embd, &len); gw_tensor(&w, N("ffn_norm.weight"), OR_F32, d, len, 1, embd, 1, 1);
        d = mat(&rng, type, ff, embd, 0.08f, &len); gw_tensor(&w, N("ffn_gate.weight"), type, d, len, 2, embd, ff, 1);
        d = mat(&rng, type, ff, embd, 0.08f, &len); gw_tensor(&w, N("ffn_up.weight"), type, d, len, 2, embd, ff, 1);
        d = mat(&rng, type, embd, ff, 0.06f, &len); gw_tensor(&w, N("ffn_down.weight"), type, d, len, 2, ff, embd, 1);
#undef N
    }
    d = normv(&rng, embd, &len); gw_tensor(&w, "output_norm.weight", OR_F32, d, len, 1, embd, 1, 1);
    if (!tied) { d = mat(&rng, type, vocab, embd, 0.08f, &len); gw_tensor(&w, "output.weight", type, d, len, 2, embd, vocab, 1); }
    int rc = gw_save(&w, path);
    gw_free(&w);
    return rc;
#undef K
}

/* C#'s default float formatting for the fixture names (round-trip shortest form, no exponent for these values). */
static void cs_float(char* out, size_t n, float v)
{
    for (int prec = 1; prec <= 9; ++prec) {
        snprintf(out, n, "%.*g", prec, (double)v);
        if ((float)strtod(out, NULL) == v) return;
    }
}

/* TinyArchs.Build (tests/TinyArchs.cs:31-106): tiny Granite and OLMo 2 models and the Llama twin of a Granite model.
 * es/rs/as/ls: the Granite scales (0 = key left out); omit_post_ffw: leave out post_ffw_norm (olmo2); short_qnorm:
 * attn_q_norm covers one head (olmo2). */
int or_write_tiny_arch(const char* path, const char* arch, int type, int tied, int layers, int embd, int heads,
                       int kv_heads, int ff, float es, float rs, float as, float ls, int omit_post_ffw, int short_qnorm,
                       uint64_t seed)
{
    or_rng rng; or_rng_init(&rng, seed);
    gw w; memset(&w, 0, sizeof w);
    char a[64], key[128], name[256];
    snprintf(a, sizeof a, "%s.", arch);
    const int olmo = strcmp(arch, "olmo2") == 0, granite = strcmp(arch, "granite") == 0;
    const int hd = embd / heads, E = embd, qd = heads * hd, kd = kv_heads * hd, F = ff;
    char scaled[160] = "";
    if (es != 0 || rs != 0 || as != 0 || ls != 0) {
        char f0[32], f1[32], f2[32], f3[32];
        cs_float(f0, sizeof f0, es); cs_float(f1, sizeof f1, rs); cs_float(f2, sizeof f2, as); cs_float(f3, sizeof f3, ls);
        snprintf(scaled, sizeof scaled, "-scaled%s_%s_%s_%s", f0, f1, f2, f3);
    }
    snprintf(name, sizeof name, "tiny-arch-%s-%s%s%s%s%s-s%llu", arch, type_name(type), tied ? "-tied" : "", scaled,
             omit_post_ffw ? "-nopost_ffw_norm" : "", short_qnorm ? "-shortq" : "", (unsigned long long)seed);
    gw_str(&w, "general.architecture", arch);
    gw_str(&w, "general.name", name);
    gw_u32(&w, "general.alignment", 32);
#define K(s) (snprintf(key, sizeof key, "%s%s", a, s), key)
    gw_u32(&w, K("block_count"), (uint32_t)layers);
    gw_u32(&w, K("context_length"), 512);
    gw_u32(&w, K("embedding_length"), (uint32_t)E);
    gw_u32(&w, K("feed_forward_length"), (uint32_t)F);
    gw_u32(&w, K("attention.head_count"), (uint32_t)heads);
    gw_u32(&w, K("attention.head_count_kv"), (uint32_t)kv_heads);
    gw_f32(&w, K("attention.layer_norm_rms_epsilon"), 1e-5f);
    gw_f32(&w, K("rope.freq_base"), 500000.0f);
    if (!olmo) gw_u32(&w, K("rope.dimension_count"), (uint32_t)hd);
    if (granite) {
        if (es != 0) gw_f32(&w, K("embedding_scale"), es);
        if (rs != 0) gw_f32(&w, K("residual_scale"), rs);
        if (as != 0) gw_f32(&w, K("attention.scale"), as);
        if (ls != 0) gw_f32(&w, K("logit_scale"), ls);
    }
#undef K
    int vocab;
    add_bpe_meta(&w, 1, &vocab);
    int64_t len; uint8_t* d;
    d = mat(&rng, type, vocab, E, 1.0f, &len); gw_tensor(&w, "token_embd.weight", type, d, len, 2, E, vocab, 1);
    for (int l = 0; l < layers; l++) {
        char p[32]; snprintf(p, sizeof p, "blk.%d.", l);
#define N(s) (snprintf(name, sizeof name, "%s%s", p, s), name)
        if (!olmo) { d = normv(&rng, E, &len); gw_tensor(&w, N("attn_norm.weight"), OR_F32, d, len, 1, E, 1, 1); }
        d = mat(&rng, type, qd, E, 0.08f, &len); gw_tensor(&w, N("attn_q.weight"), type, d, len, 2, E, qd, 1);
        d = mat(&rng, type, kd, E, 0.08f, &len); gw_tensor(&w, N("attn_k.weight"), type, d, len, 2, E, kd, 1);
        d = mat(&rng, type, kd, E, 0.08f, &len); gw_tensor(&w, N("attn_v.weight"), type, d, len, 2, E, kd, 1);
        if (olmo) {
            const int qn = short_qnorm ? hd : qd;
            d = normv(&rng, qn, &len); gw_tensor(&w, N("attn_q_norm.weight"), OR_F32, d, len, 1, qn, 1, 1);
            d = normv(&rng, kd, &len); gw_tensor(&w, N("attn_k_norm.weight"), OR_F32, d, len, 1, kd, 1, 1);
        }
        d = mat(&rng, type, E, qd, 0.08f, &len); gw_tensor(&w, N("attn_output.weight"), type, d, len, 2, qd, E, 1);
        if (olmo) { d = normv(&rng, E, &len); gw_tensor(&w, N("post_attention_norm.weight"), OR_F32, d, len, 1, E, 1, 1); }
        else { d = normv(&rng, E, &len); gw_tensor(&w, N("ffn_norm.weight"), OR_F32, d, len, 1, E, 1, 1); }
        d = mat(&rng, type, F, E, 0.08f, &len); gw_tensor(&w, N("ffn_gate.weight"), type, d, len, 2, E, F, 1);
        d = mat(&rng, type, F, E, 0.08f, &len); gw_tensor(&w, N("ffn_up.weight"), type, d, len, 2, E, F, 1);
        d = mat(&rng, type, E, F, 0.06f, &len); gw_tensor(&w, N("ffn_down.weight"), type, d, len, 2, F, E, 1);
        if (olmo && !omit_post_ffw) { d = normv(&rng, E, &len); gw_tensor(&w, N("post_ffw_norm.weight"), OR_F32, d, len, 1, E, 1, 1); }
#undef N
    }
    d = normv(&rng, E, &len); gw_tensor(&w, "output_norm.weight", OR_F32, d, len, 1, E, 1, 1);
    if (!tied) { d = mat(&rng, type, vocab, E, 0.08f, &len); gw_tensor(&w, "output.weight", type, d, len, 2, E, vocab, 1); }
    int rc = gw_save(&w, path);
    gw_free(&w);
    return rc;
}

/* TinyMoe.Build (tests/TinyMoe.cs:51-153). */
int or_write_tiny_moe(const char* path, const char* layout, int ty, int tied, int layers, int E, int heads, int kv_heads,
                      int experts, int used, int X, int SH, int DF, int norm_key, uint32_t dense_mask, int dense_twin, uint64_t seed)
{
    int qwen = strcmp(layout, "qwen2moe") == 0 || strcmp(layout, "qwen3moe") == 0;
    const char* arch = dense_twin ? (strcmp(layout, "qwen3moe") == 0 ? "qwen3" : strcmp(layout, "qwen2moe") == 0 ? "qwen2" : "llama") : layout;
    or_rng rng; or_rng_init(&rng, seed);
    gw w; memset(&w, 0, sizeof w);
    char a[64], key[128], name[160];
    snprintf(a, sizeof a, "%s.", arch);
    int hd = E / heads;
    gw_str(&w, "general.architecture", arch);
    gw_str(&w, "general.name", "tiny-moe");
    gw_u32(&w, "general.alignment", 32);
#define K(s) (snprintf(key, sizeof key, "%s%s", a, s), key)
    gw_u32(&w, K("block_count"), (uint32_t)layers);
    gw_u32(&w, K("context_length"), 512);
    gw_u32(&w, K("embedding_length"), (uint32_t)E);
    gw_u32(&w, K("feed_forward_length"), (uint32_t)DF);
    gw_u32(&w, K("attention.head_count"), (uint32_t)heads);
    gw_u32(&w, K("attention.head_count_kv"), (uint32_t)kv_heads);
    gw_f32(&w, K("attention.layer_norm_rms_epsilon"), 1e-5f);
    gw_f32(&w, K("rope.freq_base"), qwen ? 1000000.0f : 500000.0f);
    if (strcmp(arch, "qwen3") == 0 || strcmp(arch, "qwen3moe") == 0) { gw_u32(&w, K("attention.key_length"), (uint32_t)hd); gw_u32(&w, K("attention.value_length"), (uint32_t)hd); }
    if (!qwen) gw_u32(&w, K("rope.dimension_count"), (uint32_t)hd);
    if (!dense_twin) {
        gw_u32(&w, K("expert_count"), (uint32_t)experts);
        gw_u32(&w, K("expert_used_count"), (uint32_t)used);
        gw_u32(&w, K("expert_feed_forward_length"), (uint32_t)X);
        if (strcmp(layout, "qwen2moe") == 0) gw_u32(&w, K("expert_shared_feed_forward_length"), (uint32_t)SH);
        if (norm_key >= 0) gw_bool(&w, K("expert_weights_norm"), norm_key == 1);
    }
#undef K
    int vocab; add_bpe_meta(&w, !qwen, &vocab);
    int qd = heads * hd, kd = kv_heads * hd;
    int64_t len; uint8_t* d;
    int is_q2 = strcmp(arch, "qwen2") == 0 || strcmp(arch, "qwen2moe") == 0;
    int is_q3 = strcmp(arch, "qwen3") == 0 || strcmp(arch, "qwen3moe") == 0;
    d = mat(&rng, ty, vocab, E, 1.0f, &len); gw_tensor(&w, "token_embd.weight", ty, d, len, 2, E, vocab, 1);
    for (int l = 0; l < layers; l++) {
        char p[32]; snprintf(p, sizeof p, "blk.%d.", l);
#define N(s) (snprintf(name, sizeof name, "%s%s", p, s), name)
        d = normv(&rng, E, &len); gw_tensor(&w, N("attn_norm.weight"), OR_F32, d, len, 1, E, 1, 1);
        d = mat(&rng, ty, qd, E, 0.08f, &len); gw_tensor(&w, N("attn_q.weight"), ty, d, len, 2, E, qd, 1);
        d = mat(&rng, ty, kd, E, 0.08f, &len); gw_tensor(&w, N("attn_k.weight"), ty, d, len, 2, E, kd, 1);
        d = mat(&rng, ty, kd, E, 0.08f, &len); gw_tensor(&w, N("attn_v.weight"), ty, d, len, 2, E, kd, 1);
        if (is_q2) {
            d = vecv(&rng, qd, 0.1f, &len); gw_tensor(&w, N("attn_q.bias"), OR_F32, d, len, 1, qd, 1, 1);
            d = vecv(&rng, kd, 0.1f, &len); gw_tensor(&w, N("attn_k.bias"), OR_F32, d, len, 1, kd, 1, 1);
            d = vecv(&rng, kd, 0.1f, &len); gw_tensor(&w, N("attn_v.bias"), OR_F32, d, len, 1, kd, 1, 1);
        }
        if (is_q3) {
            d = normv(&rng, hd, &len); gw_tensor(&w, N("attn_q_norm.weight"), OR_F32, d, len, 1, hd, 1, 1);
            d = normv(&rng, hd, &len); gw_tensor(&w, N("attn_k_norm.weight"), OR_F32, d, len, 1, hd, 1, 1);
        }
        d = mat(&rng, ty, E, qd, 0.08f, &len); gw_tensor(&w, N("attn_output.weight"), ty, d, len, 2, qd, E, 1);
        d = normv(&rng, E, &len); gw_tensor(&w, N("ffn_norm.weight"), OR_F32, d, len, 1, E, 1, 1);
        if ((dense_mask >> l) & 1) {
            d = mat(&rng, ty, DF, E, 0.08f, &len); gw_tensor(&w, N("ffn_gate.weight"), ty, d, len, 2, E, DF, 1);
            d = mat(&rng, ty, DF, E, 0.08f, &len); gw_tensor(&w, N("ffn_up.weight"), ty, d, len, 2, E, DF, 1);
            d = mat(&rng, ty, E, DF, 0.06f, &len); gw_tensor(&w, N("ffn_down.weight"), ty, d, len, 2, DF, E, 1);
            continue;
        }
        int64_t lr, lg, lu, ld;
        uint8_t* router = mat(&rng, OR_F32, experts, E, 0.1f, &lr);
        uint8_t* gate = mat(&rng, ty, experts * X, E, 0.08f, &lg);
        uint8_t* up = mat(&rng, ty, experts * X, E, 0.08f, &lu);
        uint8_t* down = mat(&rng, ty, experts * E, X, 0.06f, &ld);
        if (dense_twin) {
            free(router);
            gw_tensor(&w, N("ffn_gate.weight"), ty, gate, lg, 2, E, X, 1);
            gw_tensor(&w, N("ffn_up.weight"), ty, up, lu, 2, E, X, 1);
            gw_tensor(&w, N("ffn_down.weight"), ty, down, ld, 2, X, E, 1);
            continue;
        }
        gw_tensor(&w, N("ffn_gate_inp.weight"), OR_F32, router, lr, 2, E, experts, 1);
        gw_tensor(&w, N("ffn_gate_exps.weight"), ty, gate, lg, 3, E, X, experts);
        gw_tensor(&w, N("ffn_up_exps.weight"), ty, up, lu, 3, E, X, experts);
        gw_tensor(&w, N("ffn_down_exps.weight"), ty, down, ld, 3, X, E, experts);
        if (strcmp(layout, "qwen2moe") == 0) {
            d = vecv(&rng, E, 0.2f, &len); gw_tensor(&w, N("ffn_gate_inp_shexp.weight"), OR_F32, d, len, 1, E, 1, 1);
            d = mat(&rng, ty, SH, E, 0.08f, &len); gw_tensor(&w, N("ffn_gate_shexp.weight"), ty, d, len, 2, E, SH, 1);
            d = mat(&rng, ty, SH, E, 0.08f, &len); gw_tensor(&w, N("ffn_up_shexp.weight"), ty, d, len, 2, E, SH, 1);
            d = mat(&rng, ty, E, SH, 0.06f, &len); gw_tensor(&w, N("ffn_down_shexp.weight"), ty, d, len, 2, SH, E, 1);
        }
#undef N
    }
    d = normv(&rng, E, &len); gw_tensor(&w, "output_norm.weight", OR_F32, d, len, 1, E, 1, 1);
    if (!tied) { d = mat(&rng, ty, vocab, E, 0.08f, &len); gw_tensor(&w, "output.weight", ty, d, len, 2, E, vocab, 1); }
    int rc = gw_save(&w, path);
    gw_free(&w);
    return rc;
}

/* ---------------- round-to-nearest quantizers (this repository's own, for N(0, sigma) synthetic weights) ---------------- */
static inline float rnd(float v) { return rintf(v); }
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

/* Q8_0: d = fp16(max|x|/127); q = rint(x/d). */
static void quant_q8_0(const float* x, uint8_t* out)
{
    float amax = 0;
    for (int j = 0; j < 32; j++) { float a = fabsf(x[j]); if (a > amax) amax = a; }
    uint16_t dh = or_float_to_half(amax / 127.0f);
    float d = or_half_to_float(dh);
    out[0] = (uint8_t)dh; out[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 32; j++) out[2 + j] = (uint8_t)(int8_t)(d != 0.0f ? clampi((int)rnd(x[j] / d), -127, 127) : 0);
}

/* Q4_K: per 32-value sub-block an offset m = -min(0, min x) and a step (max x + m)/15; the superblock stores
 * fp16 d = max step/63 and dmin = max m/63 with 6-bit multipliers; q = rint((x + dmin*mq)/(d*sq)) in 0..15. */
static void quant_q4_k(const float* x, uint8_t* out)
{
    float step[8], off[8];
    for (int j = 0; j < 8; j++) {
        float lo = 0, hi = 0;
        for (int l = 0; l < 32; l++) { float v = x[32 * j + l]; if (v < lo) lo = v; if (v > hi) hi = v; }
        off[j] = -lo;
        step[j] = (hi - lo) / 15.0f;
    }
    float smax = 0, mmax = 0;
    for (int j = 0; j < 8; j++) { if (step[j] > smax) smax = step[j]; if (off[j] > mmax) mmax = off[j]; }
    uint16_t dh = or_float_to_half(smax / 63.0f), mh = or_float_to_half(mmax / 63.0f);
    float d = or_half_to_float(dh), dmin = or_half_to_float(mh);
    int sq[8], mq[8];
    for (int j = 0; j < 8; j++) {
        sq[j] = d != 0.0f ? clampi((int)rnd(step[j] / d), 0, 63) : 0;
        mq[j] = dmin != 0.0f ? clampi((int)rnd(off[j] / dmin), 0, 63) : 0;
    }
    memset(out, 0, 144);
    out[0] = (uint8_t)dh; out[1] = (uint8_t)(dh >> 8); out[2] = (uint8_t)mh; out[3] = (uint8_t)(mh >> 8);
    uint8_t* sc = out + 4;
    for (int j = 0; j < 4; j++) {
        sc[j] = (uint8_t)((sq[j] & 63) | ((sq[j + 4] >> 4) << 6));
        sc[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
        sc[j + 8] = (uint8_t)((sq[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
    }
    uint8_t* qs = out + 16;
    for (int pair = 0; pair < 4; pair++) {
        for (int h = 0; h < 2; h++) {
            int j = 2 * pair + h;
            float dj = d * (float)sq[j], mj = dmin * (float)mq[j];
            for (int l = 0; l < 32; l++) {
                int q = dj != 0.0f ? clampi((int)rnd((x[32 * j + l] + mj) / dj), 0, 15) : 0;
                qs[32 * pair + l] |= (uint8_t)(q << (4 * h));
            }
        }
    }
}

/* Q6_K: per 16-value group a step max|x|/32 stored as an int8 multiple of fp16 d = max step/127;
 * q = rint(x/(d*sc)) in -32..31, stored +32 in 6 bits (4 low bits in ql, 2 high in qh). */
static void quant_q6_k(const float* x, uint8_t* out)
{
    float step[16];
    for (int g = 0; g < 16; g++) {
        float amax = 0;
        for (int l = 0; l < 16; l++) { float a = fabsf(x[16 * g + l]); if (a > amax) amax = a; }
        step[g] = amax / 32.0f;
    }
    float smax = 0;
    for (int g = 0; g < 16; g++) if (step[g] > smax) smax = step[g];
    uint16_t dh = or_float_to_half(smax / 127.0f);
    float d = or_half_to_float(dh);
    int sc[16];
    for (int g = 0; g < 16; g++) sc[g] = d != 0.0f ? clampi((int)rnd(step[g] / d), -128, 127) : 0;
    memset(out, 0, 210);
    uint8_t* ql = out; uint8_t* qh = out + 128; int8_t* scs = (int8_t*)(out + 192);
    for (int g = 0; g < 16; g++) scs[g] = (int8_t)sc[g];
    out[208] = (uint8_t)dh; out[209] = (uint8_t)(dh >> 8);
    for (int e = 0; e < 256; e++) {
        float dg = d * (float)sc[e / 16];
        int q = dg != 0.0f ? clampi((int)rnd(x[e] / dg), -32, 31) : 0;
        int u = q + 32;
        int half = e / 128, w = e % 128, l = w % 32, quarter = w / 32;   /* quarter: 0 lo ql[l], 1 lo ql[l+32], 2 hi ql[l], 3 hi ql[l+32] */
        uint8_t* qlh = ql + 64 * half; uint8_t* qhh = qh + 32 * half;
        int qli = (quarter & 1) ? l + 32 : l;
        qlh[qli] |= (uint8_t)((u & 0xF) << ((quarter >> 1) * 4));
        qhh[l] |= (uint8_t)(((u >> 4) & 3) << (2 * quarter));
    }
}

void or_quantize_block(int type, const float* x, uint8_t* out)
{
    switch (type) {
    case OR_Q8_0: quant_q8_0(x, out); break;
    case OR_Q4_K: quant_q4_k(x, out); break;
    case OR_Q6_K: quant_q6_k(x, out); break;
    }
}

/* ---------------- counter-based synthetic weights ---------------- */
static inline uint64_t splitmix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* Irwin-Hall(12) over 16-bit uniforms: S - 393210 is an integer with |S - 393210| < 2^19, so the scaled value is
 * exact in float before the single multiply by sigma. */
static inline float synth_normal(uint64_t base, int64_t i)
{
    uint64_t h0 = splitmix64(base + 3 * (uint64_t)i), h1 = splitmix64(base + 3 * (uint64_t)i + 1), h2 = splitmix64(base + 3 * (uint64_t)i + 2);
    int64_t s = 0;
    for (int k = 0; k < 4; k++) s += (int64_t)((h0 >> (16 * k)) & 0xFFFF) + (int64_t)((h1 >> (16 * k)) & 0xFFFF) + (int64_t)((h2 >> (16 * k)) & 0xFFFF);
    return (float)(s - 393210) * (1.0f / 65536.0f);
}

typedef struct { int type; uint64_t base; int64_t rows, cols; float sigma, offset; uint8_t* out; int bs, ts; } synth_ctx;

static void synth_task(void* vctx, int64_t begin, int64_t end)
{
    synth_ctx* c = (synth_ctx*)vctx;
    float x[256];
    int64_t bpr = c->cols / c->bs;
    for (int64_t b = begin; b < end; b++) {
        int64_t e0 = b * c->bs;
        if (c->type == OR_F32) {
            float v = c->offset + c->sigma * synth_normal(c->base, e0);
            memcpy(c->out + b * 4, &v, 4);
            continue;
        }
        if (c->type == OR_F16) {
            uint16_t h = or_float_to_half(c->sigma * synth_normal(c->base, e0));
            memcpy(c->out + b * 2, &h, 2);
            continue;
        }
        for (int j = 0; j < c->bs; j++) x[j] = c->sigma * synth_normal(c->base, e0 + j);
        or_quantize_block(c->type, x, c->out + b * c->ts);
        (void)bpr;
    }
}

uint64_t or_synth_base(uint64_t seed, uint32_t tid) { return splitmix64(seed ^ ((uint64_t)tid * 0xD1B54A32D192ED03ULL)); }

int or_synth_tensor(int type, uint64_t seed, uint32_t tid, int64_t rows, int64_t cols, float sigma, float offset, uint8_t* out,
                    int threads)
{
    if (type != OR_F32 && type != OR_F16 && type != OR_Q8_0 && type != OR_Q4_K && type != OR_Q6_K) return -1;
    synth_ctx c;
    c.type = type; c.base = or_synth_base(seed, tid); c.rows = rows; c.cols = cols; c.sigma = sigma; c.offset = offset; c.out = out;
    or_layout(type, &c.bs, &c.ts);
    if (cols % c.bs) return -1;
    or_parallel_for(rows * cols / c.bs, threads, synth_task, &c);
    return 0;
}

/* ---------------- synthetic decoders of the benchmark configurations ---------------- */
static void synth_add(or_gguf* g, const char* name, int type, int nd, int64_t d0, int64_t d1, int64_t d2, uint32_t tid,
                      const or_synth_spec* s, float offset, int threads)
{
    int bs, ts; or_layout(type, &bs, &ts);
    int64_t rows = d1 * d2, cols = d0;
    int64_t size = rows * cols / bs * ts;
    uint8_t* data = (uint8_t*)malloc((size_t)size);
    float sigma = s->sigma > 0 ? s->sigma : 0.02f;
    or_synth_tensor(type, s->seed, tid, rows, cols, sigma, offset, data, threads);
    int64_t dims[3] = { d0, d1, d2 };
    or_gguf_mem_add_tensor(g, name, type, nd, dims, data, size);
}

or_gguf* or_synth_gguf(const or_synth_spec* s, int build_layers, int threads)
{
    int moe = strcmp(s->arch, "qwen3moe") == 0, qwen = strcmp(s->arch, "llama") != 0;
    if (strcmp(s->arch, "llama") && strcmp(s->arch, "qwen3") && strcmp(s->arch, "qwen3moe")) return NULL;
    int L = build_layers > 0 && build_layers < s->layers ? build_layers : s->layers;
    int hd = s->head_dim > 0 ? s->head_dim : s->embd / s->heads;
    int E = s->embd, QD = s->heads * hd, KD = s->kv_heads * hd, F = s->ff, NE = s->experts, X = s->expert_ff;
    or_gguf* g = or_gguf_mem_new();
    char k[160], n[160];
#define KEY(x) (snprintf(k, sizeof k, "%s.%s", s->arch, x), k)
    or_gguf_mem_set_string(g, "general.architecture", s->arch);
    or_gguf_mem_set_string(g, "general.name", "windlass-synthetic");
    or_gguf_mem_set_int(g, "general.alignment", 32);
    or_gguf_mem_set_int(g, KEY("block_count"), L);
    or_gguf_mem_set_int(g, KEY("context_length"), s->context_length > 0 ? s->context_length : 4096);
    or_gguf_mem_set_int(g, KEY("embedding_length"), E);
    or_gguf_mem_set_int(g, KEY("feed_forward_length"), F);
    or_gguf_mem_set_int(g, KEY("attention.head_count"), s->heads);
    or_gguf_mem_set_int(g, KEY("attention.head_count_kv"), s->kv_heads);
    or_gguf_mem_set_int(g, KEY("attention.key_length"), hd);
    or_gguf_mem_set_int(g, KEY("attention.value_length"), hd);
    or_gguf_mem_set_int(g, KEY("rope.dimension_count"), hd);
    or_gguf_mem_set_float(g, KEY("attention.layer_norm_rms_epsilon"), s->rms_eps > 0 ? s->rms_eps : 1e-5f);
    or_gguf_mem_set_float(g, KEY("rope.freq_base"), s->rope_base > 0 ? s->rope_base : 10000.0f);
    if (moe) {
        or_gguf_mem_set_int(g, KEY("expert_count"), NE);
        or_gguf_mem_set_int(g, KEY("expert_used_count"), s->experts_used);
        or_gguf_mem_set_int(g, KEY("expert_feed_forward_length"), X);
    }
#undef KEY
    synth_add(g, "token_embd.weight", s->type_embd, 2, E, s->vocab, 1, 1, s, 0.0f, threads);
    for (int l = 0; l < L; l++) {
        uint32_t b = (uint32_t)(l + 1) << 8;
#define NM(x) (snprintf(n, sizeof n, "blk.%d.%s", l, x), n)
        synth_add(g, NM("attn_norm.weight"), OR_F32, 1, E, 1, 1, b | 1, s, 1.0f, threads);
        synth_add(g, NM("attn_q.weight"), s->type_attn, 2, E, QD, 1, b | 2, s, 0.0f, threads);
        synth_add(g, NM("attn_k.weight"), s->type_attn, 2, E, KD, 1, b | 3, s, 0.0f, threads);
        synth_add(g, NM("attn_v.weight"), s->type_attn_v, 2, E, KD, 1, b | 4, s, 0.0f, threads);
        if (qwen) {
            synth_add(g, NM("attn_q_norm.weight"), OR_F32, 1, hd, 1, 1, b | 10, s, 1.0f, threads);
            synth_add(g, NM("attn_k_norm.weight"), OR_F32, 1, hd, 1, 1, b | 11, s, 1.0f, threads);
        }
        synth_add(g, NM("attn_output.weight"), s->type_attn, 2, QD, E, 1, b | 5, s, 0.0f, threads);
        synth_add(g, NM("ffn_norm.weight"), OR_F32, 1, E, 1, 1, b | 6, s, 1.0f, threads);
        if (moe) {
            synth_add(g, NM("ffn_gate_inp.weight"), OR_F32, 2, E, NE, 1, b | 12, s, 0.0f, threads);
            synth_add(g, NM("ffn_gate_exps.weight"), s->type_ffn, 3, E, X, NE, b | 13, s, 0.0f, threads);
            synth_add(g, NM("ffn_up_exps.weight"), s->type_ffn, 3, E, X, NE, b | 14, s, 0.0f, threads);
            synth_add(g, NM("ffn_down_exps.weight"), s->type_ffn_down, 3, X, E, NE, b | 15, s, 0.0f, threads);
        } else {
            synth_add(g, NM("ffn_gate.weight"), s->type_ffn, 2, E, F, 1, b | 7, s, 0.0f, threads);
            synth_add(g, NM("ffn_up.weight"), s->type_ffn, 2, E, F, 1, b | 8, s, 0.0f, threads);
            synth_add(g, NM("ffn_down.weight"), s->type_ffn_down, 2, F, E, 1, b | 9, s, 0.0f, threads);
        }
#undef NM
    }
    synth_add(g, "output_norm.weight", OR_F32, 1, E, 1, 1, 2, s, 1.0f, threads);
    synth_add(g, "output.weight", s->type_output, 2, E, s->vocab, 1, 3, s, 0.0f, threads);
    return g;
}
