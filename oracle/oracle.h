/* CPU oracle for the Windlass quantized transformer forward: test infrastructure, not product code.
 *
 * A plain-C restatement of the reference engine's CPU path (C#, .NET Framework 4.8), written to reproduce its
 * float/double evaluation order so its results are the reference's results on the same GGUF bytes:
 *   Half.cs (whole), Quants.cs:32-396, IQuants.cs:27-278, FastMath.cs:218-264 (Block), Transformer.cs (whole),
 *   ModelConfig.cs:38-155, Gguf.cs:30-66,143-208, LayerStream.cs:182-203,235-254, Engine.cs:356-360 (greedy),
 *   and the test fixtures tests/TinyModels.cs:11-97,204-381 and tests/TinyMoe.cs:51-153 (model generators).
 * Compiled with -ffp-contract=off so no multiply-add is fused (C# x64 evaluates float ops one at a time in SSE).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this library, and only as the
 * checker or the timed CPU baseline. The CUDA product never links it.
 */
#ifndef WINDLASS_ORACLE_H
#define WINDLASS_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type numbers (Gguf.cs:19-25). */
enum {
    OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q5_0 = 6, OR_Q5_1 = 7, OR_Q8_0 = 8, OR_Q8_1 = 9,
    OR_Q2_K = 10, OR_Q3_K = 11, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14, OR_Q8_K = 15,
    OR_IQ2_XXS = 16, OR_IQ2_XS = 17, OR_IQ3_XXS = 18, OR_IQ1_S = 19, OR_IQ4_NL = 20, OR_IQ3_S = 21,
    OR_IQ2_S = 22, OR_IQ4_XS = 23, OR_I8 = 24, OR_I16 = 25, OR_I32 = 26, OR_I64 = 27, OR_F64 = 28,
    OR_IQ1_M = 29, OR_BF16 = 30
};

/* ---- numerics (or_quants.c) ---- */
float    or_half_to_float(uint16_t h);                 /* Half.Decode, Half.cs:59-89 */
uint16_t or_float_to_half(float f);                    /* Half.FromFloat, Half.cs:29-57 */
int      or_layout(int type, int* block, int* bytes);  /* GgmlTypes.TryGetLayout, Gguf.cs:30-66 */
int      or_can_decode(int type);                      /* Quants.CanDecode, Quants.cs:11-21 */
int      or_can_dot(int type);                         /* Quants.CanDot, Quants.cs:56-65 */
int      or_decode_row(int type, const uint8_t* src, int64_t n, float* dst);    /* Quants.DecodeRow */
float    or_dot_row(int type, const uint8_t* b, const float* x, int n);         /* Quants.DotRow */
void     or_block(const float* w, int ws, int nr, const float* x, int xs, int nt, int cols, float* y, int ystride);
float    or_dot_f32(const float* a, const float* b, int n);                      /* Transformer.Dot */

/* y[t*rows + r] = W[r] . x[t]  (Transformer.MatMul / MatMulEach, Transformer.cs:483-561). each_token selects
 * MatMulEach (ForwardBatch). threads = worker count (0 = all cores). Returns 0 or -1 on a bad type. */
int or_matmul(int type, const uint8_t* w, int rows, int cols, int64_t row_bytes, const float* x, int T,
              float* y, int each_token, int threads);

/* ---- thread pool (or_pool.c) ---- */
typedef void (*or_task_fn)(void* ctx, int64_t begin, int64_t end);
void or_parallel_for(int64_t n, int threads, or_task_fn fn, void* ctx);
int  or_default_threads(void);

/* ---- GGUF (or_gguf.c) ---- */
typedef struct or_gguf or_gguf;
or_gguf*    or_gguf_open(const char* path, char* err, int errlen);   /* GgufModelFile.Open (one file) */
void        or_gguf_close(or_gguf* g);
int         or_gguf_tensor_count(const or_gguf* g);
const char* or_gguf_tensor_name(const or_gguf* g, int i);
int         or_gguf_find(const or_gguf* g, const char* name);          /* index or -1 */
int         or_gguf_tensor_info(const or_gguf* g, int i, int* type, int64_t dims[4], int* ndims,
                                int64_t* size_bytes, const uint8_t** data);
int         or_gguf_has(const or_gguf* g, const char* key);
int64_t     or_gguf_get_int(const or_gguf* g, const char* key, int64_t dflt);
float       or_gguf_get_float(const or_gguf* g, const char* key, float dflt);
const char* or_gguf_get_string(const or_gguf* g, const char* key, const char* dflt);
int         or_gguf_get_bool(const or_gguf* g, const char* key, int dflt);
/* In-memory GGUF whose tensors own their bytes (synthetic models that never touch the disk). */
or_gguf*    or_gguf_mem_new(void);
void        or_gguf_mem_set_int(or_gguf* g, const char* key, int64_t v);
void        or_gguf_mem_set_float(or_gguf* g, const char* key, float v);
void        or_gguf_mem_set_string(or_gguf* g, const char* key, const char* v);
void        or_gguf_mem_add_tensor(or_gguf* g, const char* name, int type, int nd, const int64_t* dims, uint8_t* data,
                                   int64_t size);

/* A synthetic decoder of the benchmark configurations, with the tensor ids the CUDA library's wl_open_synthetic
 * uses: (layer+1)<<8 | slot for layer tensors (slots 1 attn_norm, 2 q, 3 k, 4 v, 5 o, 6 ffn_norm, 7 gate, 8 up,
 * 9 down, 10 q_norm, 11 k_norm, 12 router, 13 gate_exps, 14 up_exps, 15 down_exps), 1 token_embd, 2 output_norm,
 * 3 output. Norm weights are 1 + sigma*z. arch: llama | qwen3 | qwen3moe. build_layers < layers builds only the first
 * build_layers layers (the metadata still says build_layers). */
typedef struct {
    char arch[16];
    int layers, embd, heads, kv_heads, head_dim, ff, vocab, context_length, experts, experts_used, expert_ff;
    float rope_base, rms_eps, sigma;
    int type_attn, type_attn_v, type_ffn, type_ffn_down, type_embd, type_output;
    uint64_t seed;
} or_synth_spec;
or_gguf* or_synth_gguf(const or_synth_spec* s, int build_layers, int threads);
/* Writes an in-memory GGUF (for example a synthetic model) to a file. */
int      or_gguf_save(const or_gguf* g, const char* path);

/* ---- generators (or_gen.c): the reference's test-fixture models and the synthetic benchmark weights ---- */
typedef struct { uint64_t s; } or_rng;
void     or_rng_init(or_rng* r, uint64_t seed);       /* tests/TinyModels.cs:89-97 */
uint64_t or_rng_next(or_rng* r);
uint8_t  or_rng_byte(or_rng* r);
double   or_rng_uniform(or_rng* r);
float    or_rng_normal(or_rng* r);
/* TinyModels.Matrix (tests/TinyModels.cs:344-381): random block bytes with fitted fp16 scales. out must hold
 * rows*cols/block*bytes bytes. */
int  or_matrix(or_rng* r, int type, int rows, int cols, float rms, uint8_t* out);
/* TinyModels.Build + GgufWriter.Save: writes the fixture model. arch: llama|qwen2|qwen3; flags: 1 tied, 2 spm,
 * 4 rope_freqs. Returns 0 or -1. */
int  or_write_tiny(const char* path, const char* arch, int type, int flags, int layers, int embd, int heads,
                   int kv_heads, int ff, uint64_t seed);
/* TinyArchs.Build (tests/TinyArchs.cs:31-106): arch granite | olmo2 | llama (the Granite twin); the Granite scales
 * (0 = key left out), omit_post_ffw and short_qnorm make the OLMo 2 files the reference must refuse. */
int  or_write_tiny_arch(const char* path, const char* arch, int type, int tied, int layers, int embd, int heads,
                        int kv_heads, int ff, float es, float rs, float as, float ls, int omit_post_ffw, int short_qnorm,
                        uint64_t seed);
/* TinyMoe.Build (tests/TinyMoe.cs:51-153). layout: llama|mixtral|qwen2moe|qwen3moe. dense_mask: bit l set =
 * layer l has a plain FFN. norm_key: -1 absent, 0/1 written. dense_twin: write the one-expert dense twin. */
int  or_write_tiny_moe(const char* path, const char* layout, int type, int tied, int layers, int embd, int heads,
                       int kv_heads, int experts, int used, int expert_ff, int shared_ff, int dense_ff,
                       int norm_key, uint32_t dense_mask, int dense_twin, uint64_t seed);

/* Synthetic benchmark weights, shared bit-for-bit with the CUDA generator: element i of tensor `tid` is an
 * Irwin-Hall(12) normal z drawn from a counter hash of (seed, tid, i); quantized types round-to-nearest quantize
 * sigma*z one block at a time, F32 tensors store offset + sigma*z (offset 1 for norm weights). */
int  or_synth_tensor(int type, uint64_t seed, uint32_t tid, int64_t rows, int64_t cols, float sigma, float offset,
                     uint8_t* out, int threads);
/* Round-to-nearest quantizers of one block (used by or_synth_tensor and by the config sweeps). */
void or_quantize_block(int type, const float* x, uint8_t* out);

/* ---- model (or_model.c): Transformer.cs restated ---- */
typedef struct or_model or_model;
typedef struct or_seq or_seq;
typedef struct {
    int layers, embd, heads, kv_heads, head_dim, vocab, context_length, rope_dims;
    float rms_eps, rope_base, rope_freq_scale;
    int rope_neox, qk_norm, qk_norm_full, post_norms, tied;
    float embedding_scale, residual_scale, attention_scale, logit_scale;
    int expert_count, expert_used, expert_ff, shared_expert_ff, expert_weights_norm;
    char arch[32];
} or_config;

or_model* or_model_open(const char* path, int max_context, int threads, char* err, int errlen);
/* The same over an already open (or in-memory) GGUF; the model takes ownership of g. */
or_model* or_model_open_gguf(or_gguf* g, int max_context, int threads, char* err, int errlen);
void      or_model_close(or_model* m);
int       or_model_config(const or_model* m, or_config* c);
or_seq*   or_seq_new(or_model* m);
void      or_seq_free(or_seq* s);
int       or_seq_length(const or_seq* s);
void      or_seq_truncate(or_seq* s, int n);
/* Transformer.Forward (Transformer.cs:83-109). seq NULL = the model's own sequence. out holds T*V (all) or V. */
int or_forward(or_model* m, or_seq* seq, const int32_t* tokens, int T, int pos0, int all_logits, float* out,
               char* err, int errlen);
/* Transformer.ForwardBatch (Transformer.cs:132-170). out holds N*V. */
int or_forward_batch(or_model* m, or_seq* const* seqs, const int32_t* tokens, int N, float* out, char* err,
                     int errlen);
int64_t or_expert_runs(const or_model* m);
/* Transformer.Route (Transformer.cs:315-340) for one token. */
void or_route(const float* logits, int n, int k, int renorm, int32_t* sel, float* wts, int32_t* count);
/* Transformer.RmsNormRows (Transformer.cs:454-464), in place allowed. */
void or_rmsnorm_rows(const float* x, int n, int dim, const float* w, float eps, float* y);
/* Greedy pick of Sampler.Sample (Engine.cs:356-360): the first index of the largest logit. */
int or_argmax(const float* logits, int n);
/* Sampler.Sample (Engine.cs:361-380) with the generator's uniform draw passed in; *margin (optional) = the relative
 * distance of the draw (and the nucleus limit) from the nearest boundary between ids around the choice. */
int or_sample(const float* logits, int n, double temperature, double top_p, double draw, double* margin);

/* Stage-level hooks for the bounded CPU baseline: one decoder layer of the model on T rows of x (in place),
 * positions pos0.., appending to seq. Returns 0 or -1. */
int or_layer(or_model* m, int layer, float* x, int T, int pos0, or_seq* seq, char* err, int errlen);

#ifdef __cplusplus
}
#endif
#endif
