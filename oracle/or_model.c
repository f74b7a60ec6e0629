/* Oracle model: Transformer.cs restated (Forward, ForwardBatch, Layer, Attention, RoPE, RMSNorm, SwiGLU, MoE routing,
 * Head), with ModelConfig.From (ModelConfig.cs:38-155) and the stage name binding of LayerStream.Bind
 * (LayerStream.cs:182-203). Weights are read from an mmap of the GGUF file; the streaming machinery of LayerStream
 * is not restated because the reference's tests show it is exact (StreamingIsExact, tests/Tests.cs:305-321).
 * Test infrastructure only (see oracle.h). */
#include "oracle.h"
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct { int type, rows, cols, experts; int64_t row_bytes; const uint8_t* data; int present; } wview;

typedef struct {
    wview attn_norm, q, k, v, qb, kb, vb, q_norm, k_norm, o, post_attn_norm, ffn_norm, post_ffw_norm;
    wview gate, up, down, router, gate_exps, up_exps, down_exps, sh_gate_inp, sh_gate, sh_up, sh_down;
    int moe;
} layer_t;

struct or_seq { uint16_t** K; uint16_t** V; int capacity, length, layers; };

struct or_model {
    or_gguf* g;
    or_config c;
    layer_t* L;
    wview embd, out_norm, output;
    float* rope_freqs; int n_rope_freqs;
    float** rope;              /* per position cos/sin pairs, computed once */
    int max_context, threads;
    or_seq* own;
    int64_t expert_runs;
    int each_token;
};

static void seterr(char* err, int errlen, const char* msg) { if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", msg); }

static wview view_of(or_model* m, const char* name)
{
    wview v; memset(&v, 0, sizeof v);
    int i = or_gguf_find(m->g, name);
    if (i < 0) return v;
    int type, nd; int64_t dims[4], size; const uint8_t* data;
    or_gguf_tensor_info(m->g, i, &type, dims, &nd, &size, &data);
    int64_t ne = dims[0] * dims[1] * dims[2] * dims[3];
    int64_t rows_all = ne / dims[0];
    int experts = (int)(dims[2] * dims[3]);
    v.type = type; v.cols = (int)dims[0]; v.experts = experts; v.rows = (int)(rows_all / experts);
    v.row_bytes = size / rows_all; v.data = data; v.present = 1;
    return v;
}

static wview slice(const wview* w, int e)
{
    wview v = *w;
    v.experts = 1;
    v.data = w->data + (int64_t)e * w->rows * w->row_bytes;
    return v;
}

static float* vector(const wview* w)
{
    int64_t n = (int64_t)w->rows * w->cols;
    float* v = (float*)malloc(sizeof(float) * (size_t)n);
    or_decode_row(w->type, w->data, n, v);
    return v;
}

/* ModelConfig.From (ModelConfig.cs:38-110), the fields the forward reads. */
static int read_config(or_model* m, char* err, int errlen)
{
    or_gguf* g = m->g; or_config* c = &m->c;
    memset(c, 0, sizeof *c);
    const char* arch = or_gguf_get_string(g, "general.architecture", "");
    static const char* archs[] = { "llama", "qwen2", "qwen3", "mixtral", "qwen2moe", "qwen3moe", "granite", "olmo2" };
    int ok = 0;
    for (int i = 0; i < 8; i++) if (strcmp(arch, archs[i]) == 0) ok = 1;
    if (!ok) { seterr(err, errlen, "unsupported architecture"); return -1; }
    snprintf(c->arch, sizeof c->arch, "%s", arch);
    char k[160];
#define KEY(s) (snprintf(k, sizeof k, "%s.%s", arch, s), k)
    c->layers = (int)or_gguf_get_int(g, KEY("block_count"), 0);
    c->embd = (int)or_gguf_get_int(g, KEY("embedding_length"), 0);
    c->heads = (int)or_gguf_get_int(g, KEY("attention.head_count"), 0);
    c->kv_heads = (int)or_gguf_get_int(g, KEY("attention.head_count_kv"), c->heads);
    c->head_dim = (int)or_gguf_get_int(g, KEY("attention.key_length"), c->heads ? c->embd / c->heads : 0);
    c->rope_dims = (int)or_gguf_get_int(g, KEY("rope.dimension_count"), c->head_dim);
    c->context_length = (int)or_gguf_get_int(g, KEY("context_length"), 4096);
    c->rms_eps = or_gguf_get_float(g, KEY("attention.layer_norm_rms_epsilon"), 1e-5f);
    c->rope_base = or_gguf_get_float(g, KEY("rope.freq_base"), 10000.0f);
    c->rope_freq_scale = 1.0f;
    c->rope_neox = !strcmp(arch, "qwen2") || !strcmp(arch, "qwen3") || !strcmp(arch, "qwen2moe") || !strcmp(arch, "qwen3moe") || !strcmp(arch, "olmo2");
    if (!strcmp(arch, "granite")) {
        c->embedding_scale = or_gguf_get_float(g, KEY("embedding_scale"), 0);
        c->residual_scale = or_gguf_get_float(g, KEY("residual_scale"), 0);
        c->attention_scale = or_gguf_get_float(g, KEY("attention.scale"), 0);
        c->logit_scale = or_gguf_get_float(g, KEY("logit_scale"), 0);
    }
    c->post_norms = !strcmp(arch, "olmo2");
    c->qk_norm_full = !strcmp(arch, "olmo2");
    c->qk_norm = or_gguf_find(g, "blk.0.attn_q_norm.weight") >= 0;
    c->tied = or_gguf_find(g, "output.weight") < 0;
    const char* scaling = or_gguf_get_string(g, KEY("rope.scaling.type"), "none");
    float factor = or_gguf_get_float(g, KEY("rope.scaling.factor"), 0);
    if (!strcmp(scaling, "linear") && factor > 0) c->rope_freq_scale = 1.0f / factor;
    c->expert_count = (int)or_gguf_get_int(g, KEY("expert_count"), 0);
    if (c->expert_count > 0) {
        c->expert_used = (int)or_gguf_get_int(g, KEY("expert_used_count"), 0);
        if (c->expert_used < 1 || c->expert_used > c->expert_count) { seterr(err, errlen, "bad expert_used_count"); return -1; }
        int norm = strcmp(arch, "qwen2moe") != 0;
        if (or_gguf_has(g, KEY("expert_weights_norm"))) norm = or_gguf_get_bool(g, KEY("expert_weights_norm"), norm);
        c->expert_weights_norm = norm;
    } else if (!strcmp(arch, "qwen2moe") || !strcmp(arch, "qwen3moe")) { seterr(err, errlen, "MoE architecture needs expert_count"); return -1; }
#undef KEY
    if (c->layers <= 0 || c->embd <= 0 || c->heads <= 0 || c->kv_heads <= 0 || c->heads % c->kv_heads) { seterr(err, errlen, "bad model shape"); return -1; }
    if (c->rope_dims > c->head_dim || c->rope_dims % 2) { seterr(err, errlen, "unsupported rope.dimension_count"); return -1; }
    int ei = or_gguf_find(g, "token_embd.weight");
    if (ei < 0) { seterr(err, errlen, "the model has no token_embd.weight"); return -1; }
    m->embd = view_of(m, "token_embd.weight");
    c->vocab = m->embd.rows;
    return 0;
}

static int bind_layers(or_model* m, char* err, int errlen)
{
    or_config* c = &m->c;
    m->L = (layer_t*)calloc((size_t)c->layers, sizeof(layer_t));
    char n[160];
    for (int l = 0; l < c->layers; l++) {
        layer_t* L = &m->L[l];
#define V(s) (snprintf(n, sizeof n, "blk.%d.%s", l, s), view_of(m, n))
        L->attn_norm = V("attn_norm.weight"); L->q = V("attn_q.weight"); L->k = V("attn_k.weight"); L->v = V("attn_v.weight");
        L->qb = V("attn_q.bias"); L->kb = V("attn_k.bias"); L->vb = V("attn_v.bias");
        L->q_norm = V("attn_q_norm.weight"); L->k_norm = V("attn_k_norm.weight"); L->o = V("attn_output.weight");
        L->post_attn_norm = V("post_attention_norm.weight"); L->ffn_norm = V("ffn_norm.weight"); L->post_ffw_norm = V("post_ffw_norm.weight");
        L->gate = V("ffn_gate.weight"); L->up = V("ffn_up.weight"); L->down = V("ffn_down.weight");
        L->router = V("ffn_gate_inp.weight"); L->gate_exps = V("ffn_gate_exps.weight"); L->up_exps = V("ffn_up_exps.weight"); L->down_exps = V("ffn_down_exps.weight");
        L->sh_gate_inp = V("ffn_gate_inp_shexp.weight"); L->sh_gate = V("ffn_gate_shexp.weight"); L->sh_up = V("ffn_up_shexp.weight"); L->sh_down = V("ffn_down_shexp.weight");
#undef V
        L->moe = c->expert_count > 0 && L->router.present;
        if (!L->q.present || !L->k.present || !L->v.present || !L->o.present) { seterr(err, errlen, "layer is missing attention tensors"); return -1; }
        if (!c->post_norms && (!L->attn_norm.present || !L->ffn_norm.present)) { seterr(err, errlen, "layer is missing norm tensors"); return -1; }
        if (c->post_norms) {
            /* ModelConfig.Olmo2LayerTensors (src/ModelConfig.cs:115) and the whole-vector QK norm (:102-105) */
            static const char* olmo2[] = { "attn_q_norm", "attn_k_norm", "post_attention_norm", "post_ffw_norm" };
            const wview* need[] = { &L->q_norm, &L->k_norm, &L->post_attn_norm, &L->post_ffw_norm };
            for (int i = 0; i < 4; i++)
                if (!need[i]->present) {
                    char msg[160];
                    snprintf(msg, sizeof msg, "Layer %d has no %s.weight (unsupported layout).", l, olmo2[i]);
                    seterr(err, errlen, msg);
                    return -1;
                }
        }
        if (c->qk_norm_full && (L->q_norm.rows * L->q_norm.cols != c->heads * c->head_dim ||
                                L->k_norm.rows * L->k_norm.cols != c->kv_heads * c->head_dim)) {
            char msg[200];
            snprintf(msg, sizeof msg, "Layer %d: attn_q_norm/attn_k_norm must cover the whole Q and K vectors (%d and %d).", l,
                     c->heads * c->head_dim, c->kv_heads * c->head_dim);
            seterr(err, errlen, msg);
            return -1;
        }
        if (L->moe) {
            if (!L->gate_exps.present || !L->up_exps.present || !L->down_exps.present) { seterr(err, errlen, "MoE layer is missing expert tensors"); return -1; }
            c->expert_ff = L->gate_exps.rows;
            if (L->sh_gate.present) c->shared_expert_ff = L->sh_gate.rows;
        } else if (!L->gate.present || !L->up.present || !L->down.present) { seterr(err, errlen, "layer is missing FFN tensors"); return -1; }
    }
    m->out_norm = view_of(m, "output_norm.weight");
    m->output = c->tied ? m->embd : view_of(m, "output.weight");
    if (!m->out_norm.present) { seterr(err, errlen, "the model has no output_norm.weight"); return -1; }
    wview rf = view_of(m, "rope_freqs.weight");
    if (rf.present) { m->rope_freqs = vector(&rf); m->n_rope_freqs = rf.rows * rf.cols; }
    for (int i = 0; i < or_gguf_tensor_count(m->g); i++) {
        int type, nd; int64_t dims[4], size;
        or_gguf_tensor_info(m->g, i, &type, dims, &nd, &size, NULL);
        const char* nm = or_gguf_tensor_name(m->g, i);
        size_t ln = strlen(nm);
        if (ln > 7 && strcmp(nm + ln - 7, ".weight") == 0 && nd >= 2 && !or_can_decode(type)) { seterr(err, errlen, "a weight uses a type the engine cannot decode"); return -1; }
    }
    return 0;
}

or_model* or_model_open(const char* path, int max_context, int threads, char* err, int errlen)
{
    or_gguf* g = or_gguf_open(path, err, errlen);
    if (!g) return NULL;
    return or_model_open_gguf(g, max_context, threads, err, errlen);
}

or_model* or_model_open_gguf(or_gguf* g, int max_context, int threads, char* err, int errlen)
{
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    m->g = g;
    if (read_config(m, err, errlen) || bind_layers(m, err, errlen)) { or_model_close(m); return NULL; }
    m->max_context = max_context > 0 ? max_context : (m->c.context_length < 8192 ? m->c.context_length : 8192);
    m->threads = threads;
    m->rope = (float**)calloc((size_t)m->max_context, sizeof(float*));
    m->own = or_seq_new(m);
    return m;
}

void or_model_close(or_model* m)
{
    if (!m) return;
    if (m->own) or_seq_free(m->own);
    if (m->rope) { for (int i = 0; i < m->max_context; i++) free(m->rope[i]); free(m->rope); }
    free(m->rope_freqs); free(m->L);
    or_gguf_close(m->g);
    free(m);
}

int or_model_config(const or_model* m, or_config* c) { *c = m->c; return 0; }
int64_t or_expert_runs(const or_model* m) { return m->expert_runs; }

or_seq* or_seq_new(or_model* m)
{
    or_seq* s = (or_seq*)calloc(1, sizeof(or_seq));
    s->layers = m->c.layers;
    s->K = (uint16_t**)calloc((size_t)s->layers, sizeof(uint16_t*));
    s->V = (uint16_t**)calloc((size_t)s->layers, sizeof(uint16_t*));
    return s;
}
void or_seq_free(or_seq* s)
{
    if (!s) return;
    for (int l = 0; l < s->layers; l++) { free(s->K[l]); free(s->V[l]); }
    free(s->K); free(s->V); free(s);
}
int or_seq_length(const or_seq* s) { return s->length; }
/* Sequence.Truncate (Batch.cs:28). */
void or_seq_truncate(or_seq* s, int n) { if (n < s->length) s->length = n < 0 ? 0 : n; }

/* Transformer.Reserve (Transformer.cs:62-73). */
static void reserve(or_model* m, or_seq* sq, int positions)
{
    if (positions <= sq->capacity) return;
    int grow = sq->capacity * 2 > 256 ? sq->capacity * 2 : 256;
    if (grow > m->max_context) grow = m->max_context;
    int cap = positions > grow ? positions : grow;
    int64_t KD = (int64_t)m->c.kv_heads * m->c.head_dim;
    for (int l = 0; l < m->c.layers; l++) {
        uint16_t* nk = (uint16_t*)calloc((size_t)(cap * KD), 2);
        uint16_t* nv = (uint16_t*)calloc((size_t)(cap * KD), 2);
        if (sq->K[l]) { memcpy(nk, sq->K[l], (size_t)(sq->length * KD) * 2); memcpy(nv, sq->V[l], (size_t)(sq->length * KD) * 2); }
        free(sq->K[l]); free(sq->V[l]);
        sq->K[l] = nk; sq->V[l] = nv;
    }
    sq->capacity = cap;
}

/* RmsNormRows (Transformer.cs:454-464): double sum of squares, float scale. */
void or_rmsnorm_rows(const float* x, int n, int dim, const float* w, float eps, float* y)
{
    for (int r = 0; r < n; r++) {
        int64_t o = (int64_t)r * dim;
        double sum = 0;
        for (int i = 0; i < dim; i++) sum += (double)x[o + i] * x[o + i];
        float scale = 1.0f / (float)sqrt((double)((float)(sum / dim) + eps));
        for (int i = 0; i < dim; i++) y[o + i] = x[o + i] * scale * w[i];
    }
}

/* RopeTable (Transformer.cs:399-416). */
static float* rope_table(or_model* m, int pos)
{
    if (m->rope[pos]) return m->rope[pos];
    int n = m->c.rope_dims;
    float* cs = (float*)malloc(sizeof(float) * (size_t)n);
    double theta_scale = pow((double)m->c.rope_base, -2.0 / n);
    double theta = pos * (double)m->c.rope_freq_scale;
    for (int i = 0; i < n / 2; i++) {
        double t = m->rope_freqs ? theta / m->rope_freqs[i] : theta;
        cs[2 * i] = (float)cos(t);
        cs[2 * i + 1] = (float)sin(t);
        theta *= theta_scale;
    }
    m->rope[pos] = cs;
    return cs;
}

/* Rope (Transformer.cs:418-433). */
static void rope(or_model* m, float* x, int64_t offset, int heads, const float* cs)
{
    int HD = m->c.head_dim, n = m->c.rope_dims, half = n / 2;
    for (int h = 0; h < heads; h++) {
        int64_t o = offset + (int64_t)h * HD;
        for (int i = 0; i < half; i++) {
            float c = cs[2 * i], s = cs[2 * i + 1];
            int64_t a = m->c.rope_neox ? o + i : o + 2 * i, b = m->c.rope_neox ? o + i + half : o + 2 * i + 1;
            float x0 = x[a], x1 = x[b];
            x[a] = x0 * c - x1 * s;
            x[b] = x0 * s + x1 * c;
        }
    }
}

static void matmul(or_model* m, const wview* w, const float* x, int T, float* y)
{
    or_matmul(w->type, w->data, w->rows, w->cols, w->row_bytes, x, T, y, m->each_token, m->threads);
}

static void add_bias(const wview* w, float* y, int T)
{
    if (!w->present) return;
    float* b = vector(w);
    int n = w->rows * w->cols;
    for (int t = 0; t < T; t++) for (int i = 0; i < n; i++) y[(int64_t)t * n + i] += b[i];
    free(b);
}

typedef struct { or_seq** seq; int* pos; int maxn; } batch_rows;

typedef struct {
    or_model* m; int l, T, pos0; or_seq* sq; const batch_rows* br; const float* q; float* out;
} att_ctx;

/* Attention (Transformer.cs:351-395), one (token, head) job per index. */
static void att_task(void* vctx, int64_t begin, int64_t end)
{
    att_ctx* a = (att_ctx*)vctx;
    or_config* C = &a->m->c;
    int H = C->heads, HD = C->head_dim, QD = C->heads * C->head_dim, KD = C->kv_heads * C->head_dim, group = C->heads / C->kv_heads;
    float scale = C->attention_scale != 0.0f ? C->attention_scale : 1.0f / (float)sqrt((double)HD);
    int scratch = a->br == NULL ? a->pos0 + a->T : a->br->maxn;
    float* sp = (float*)malloc(sizeof(float) * (size_t)scratch);
    for (int64_t job = begin; job < end; job++) {
        int t = (int)(job / H), h = (int)(job % H), kvh = h / group;
        int n = a->br == NULL ? a->pos0 + t + 1 : a->br->pos[t] + 1;
        const uint16_t* Kp = a->br == NULL ? a->sq->K[a->l] : a->br->seq[t]->K[a->l];
        const uint16_t* Vp = a->br == NULL ? a->sq->V[a->l] : a->br->seq[t]->V[a->l];
        const float* qp = a->q + (int64_t)t * QD + h * HD;
        float mx = -INFINITY;
        for (int j = 0; j < n; j++) {
            const uint16_t* kp = Kp + (int64_t)j * KD + kvh * HD;
            float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
            int i = 0;
            for (; i + 4 <= HD; i += 4) {
                s0 += qp[i] * or_half_to_float(kp[i]); s1 += qp[i + 1] * or_half_to_float(kp[i + 1]);
                s2 += qp[i + 2] * or_half_to_float(kp[i + 2]); s3 += qp[i + 3] * or_half_to_float(kp[i + 3]);
            }
            for (; i < HD; i++) s0 += qp[i] * or_half_to_float(kp[i]);
            float d = ((s0 + s1) + (s2 + s3)) * scale;
            sp[j] = d;
            if (d > mx) mx = d;
        }
        double sum = 0;
        for (int j = 0; j < n; j++) { float e = (float)exp((double)(sp[j] - mx)); sp[j] = e; sum += e; }
        float inv = (float)(1.0 / sum);
        float* op = a->out + (int64_t)t * QD + h * HD;
        for (int d = 0; d < HD; d++) op[d] = 0;
        for (int j = 0; j < n; j++) {
            float p = sp[j] * inv;
            const uint16_t* vp = Vp + (int64_t)j * KD + kvh * HD;
            for (int d = 0; d < HD; d++) op[d] += p * or_half_to_float(vp[d]);
        }
    }
    free(sp);
}

/* SwiGlu (Transformer.cs:241-251). */
static float* swiglu(or_model* m, const wview* gate, const wview* up, const wview* down, const float* xn, int T)
{
    int F = gate->rows;
    float* g = (float*)malloc(sizeof(float) * (size_t)T * F);
    float* u = (float*)malloc(sizeof(float) * (size_t)T * F);
    matmul(m, gate, xn, T, g);
    matmul(m, up, xn, T, u);
    for (int64_t i = 0; i < (int64_t)T * F; i++) { float a = g[i]; g[i] = a / (1.0f + (float)exp(-(double)a)) * u[i]; }
    float* o = (float*)malloc(sizeof(float) * (size_t)T * down->rows);
    matmul(m, down, g, T, o);
    free(g); free(u);
    return o;
}

#define MIN_EXPERT_WEIGHT_SUM 6.103515625e-5f

/* Route (Transformer.cs:315-340). */
void or_route(const float* logits, int n, int k, int renorm, int32_t* sel, float* wts, int32_t* count)
{
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) if (logits[i] > mx) mx = logits[i];
    float* p = (float*)malloc(sizeof(float) * (size_t)n);
    double sum = 0;
    for (int i = 0; i < n; i++) { p[i] = (float)exp((double)(logits[i] - mx)); sum += p[i]; }
    float inv = (float)(1.0 / sum);
    for (int i = 0; i < n; i++) p[i] *= inv;
    uint8_t* taken = (uint8_t*)calloc((size_t)n, 1);
    float chosen = 0;
    for (int j = 0; j < k; j++) {
        int best = -1;
        for (int i = 0; i < n; i++) if (!taken[i] && (best < 0 || p[i] > p[best])) best = i;
        taken[best] = 1;
        sel[j] = best; wts[j] = p[best];
        chosen += p[best];
        if (count) count[best]++;
    }
    if (renorm) {
        float div = chosen > MIN_EXPERT_WEIGHT_SUM ? chosen : MIN_EXPERT_WEIGHT_SUM;
        for (int j = 0; j < k; j++) wts[j] /= div;
    }
    free(p); free(taken);
}

/* MoeFfn (Transformer.cs:259-311). */
static float* moe_ffn(or_model* m, layer_t* L, const float* xn, int T)
{
    int E = m->c.embd, NE = m->c.expert_count, K = m->c.expert_used;
    float* logits = (float*)malloc(sizeof(float) * (size_t)T * NE);
    matmul(m, &L->router, xn, T, logits);
    int32_t* sel = (int32_t*)malloc(sizeof(int32_t) * (size_t)T * K);
    float* wts = (float*)malloc(sizeof(float) * (size_t)T * K);
    int32_t* count = (int32_t*)calloc((size_t)NE, sizeof(int32_t));
    for (int t = 0; t < T; t++) or_route(logits + (int64_t)t * NE, NE, K, m->c.expert_weights_norm, sel + (int64_t)t * K, wts + (int64_t)t * K, count);
    float* outp = (float*)calloc((size_t)T * E, sizeof(float));
    for (int e = 0; e < NE; e++) {
        int n = count[e];
        if (n == 0) continue;
        int* toks = (int*)malloc(sizeof(int) * (size_t)n);
        float* w = (float*)malloc(sizeof(float) * (size_t)n);
        float* xe = (float*)malloc(sizeof(float) * (size_t)n * E);
        int at = 0;
        for (int t = 0; t < T; t++)
            for (int j = 0; j < K; j++)
                if (sel[(int64_t)t * K + j] == e) {
                    toks[at] = t; w[at] = wts[(int64_t)t * K + j];
                    memcpy(xe + (int64_t)at * E, xn + (int64_t)t * E, sizeof(float) * (size_t)E);
                    at++;
                }
        m->expert_runs++;
        wview g = slice(&L->gate_exps, e), u = slice(&L->up_exps, e), d = slice(&L->down_exps, e);
        float* ye = swiglu(m, &g, &u, &d, xe, n);
        for (int i = 0; i < n; i++) {
            int64_t o = (int64_t)toks[i] * E, r = (int64_t)i * E;
            for (int dd = 0; dd < E; dd++) outp[o + dd] += w[i] * ye[r + dd];
        }
        free(toks); free(w); free(xe); free(ye);
    }
    if (L->sh_gate.present) {
        float* sh = swiglu(m, &L->sh_gate, &L->sh_up, &L->sh_down, xn, T);
        float* gl = NULL;
        if (L->sh_gate_inp.present) { gl = (float*)malloc(sizeof(float) * (size_t)T); matmul(m, &L->sh_gate_inp, xn, T, gl); }
        for (int t = 0; t < T; t++) {
            float f = gl == NULL ? 1.0f : 1.0f / (1.0f + (float)exp(-(double)gl[t]));
            int64_t o = (int64_t)t * E;
            for (int dd = 0; dd < E; dd++) outp[o + dd] += f * sh[o + dd];
        }
        free(sh); free(gl);
    }
    free(logits); free(sel); free(wts); free(count);
    return outp;
}

/* Layer (Transformer.cs:177-232). br == NULL: T tokens of sq from pos0; else a batch step. */
static void layer(or_model* m, int l, float* x, int T, int pos0, or_seq* sq, const batch_rows* br)
{
    or_config* C = &m->c;
    layer_t* L = &m->L[l];
    int E = C->embd, QD = C->heads * C->head_dim, KD = C->kv_heads * C->head_dim, HD = C->head_dim;
    float rs = C->residual_scale != 0.0f ? C->residual_scale : 1.0f;
    int64_t xl = (int64_t)T * E;
    float* xn = (float*)malloc(sizeof(float) * (size_t)xl);
    if (C->post_norms) memcpy(xn, x, sizeof(float) * (size_t)xl);
    else { float* w = vector(&L->attn_norm); or_rmsnorm_rows(x, T, E, w, C->rms_eps, xn); free(w); }
    float* q = (float*)malloc(sizeof(float) * (size_t)T * QD);
    float* k = (float*)malloc(sizeof(float) * (size_t)T * KD);
    float* v = (float*)malloc(sizeof(float) * (size_t)T * KD);
    matmul(m, &L->q, xn, T, q); matmul(m, &L->k, xn, T, k); matmul(m, &L->v, xn, T, v);
    add_bias(&L->qb, q, T); add_bias(&L->kb, k, T); add_bias(&L->vb, v, T);
    if (C->qk_norm_full) {
        float* wq = vector(&L->q_norm); float* wk = vector(&L->k_norm);
        or_rmsnorm_rows(q, T, QD, wq, C->rms_eps, q); or_rmsnorm_rows(k, T, KD, wk, C->rms_eps, k);
        free(wq); free(wk);
    } else if (C->qk_norm) {
        float* wq = vector(&L->q_norm); float* wk = vector(&L->k_norm);
        or_rmsnorm_rows(q, T * C->heads, HD, wq, C->rms_eps, q); or_rmsnorm_rows(k, T * C->kv_heads, HD, wk, C->rms_eps, k);
        free(wq); free(wk);
    }
    for (int t = 0; t < T; t++) {
        float* cs = rope_table(m, br == NULL ? pos0 + t : br->pos[t]);
        rope(m, q, (int64_t)t * QD, C->heads, cs);
        rope(m, k, (int64_t)t * KD, C->kv_heads, cs);
    }
    if (br == NULL) {
        for (int64_t i = 0; i < (int64_t)T * KD; i++) {
            sq->K[l][(int64_t)pos0 * KD + i] = or_float_to_half(k[i]);
            sq->V[l][(int64_t)pos0 * KD + i] = or_float_to_half(v[i]);
        }
    } else {
        for (int t = 0; t < T; t++)
            for (int i = 0; i < KD; i++) {
                br->seq[t]->K[l][(int64_t)br->pos[t] * KD + i] = or_float_to_half(k[(int64_t)t * KD + i]);
                br->seq[t]->V[l][(int64_t)br->pos[t] * KD + i] = or_float_to_half(v[(int64_t)t * KD + i]);
            }
    }
    float* att = (float*)malloc(sizeof(float) * (size_t)T * QD);
    att_ctx ac = { m, l, T, pos0, sq, br, q, att };
    or_parallel_for((int64_t)T * C->heads, m->threads, att_task, &ac);
    float* o = (float*)malloc(sizeof(float) * (size_t)xl);
    matmul(m, &L->o, att, T, o);
    if (C->post_norms) { float* w = vector(&L->post_attn_norm); or_rmsnorm_rows(o, T, E, w, C->rms_eps, o); free(w); }
    for (int64_t i = 0; i < xl; i++) x[i] += o[i] * rs;
    free(o);
    if (C->post_norms) memcpy(xn, x, sizeof(float) * (size_t)xl);
    else { float* w = vector(&L->ffn_norm); or_rmsnorm_rows(x, T, E, w, C->rms_eps, xn); free(w); }
    o = L->moe ? moe_ffn(m, L, xn, T) : swiglu(m, &L->gate, &L->up, &L->down, xn, T);
    if (C->post_norms) { float* w = vector(&L->post_ffw_norm); or_rmsnorm_rows(o, T, E, w, C->rms_eps, o); free(w); }
    for (int64_t i = 0; i < xl; i++) x[i] += o[i] * rs;
    free(o); free(xn); free(q); free(k); free(v); free(att);
}

/* Head (Transformer.cs:112-125): final norm and output matrix for rows first..T-1. */
static void head(or_model* m, const float* x, int T, int first, float* logits)
{
    int E = m->c.embd, n = T - first;
    float* xn = (float*)malloc(sizeof(float) * (size_t)n * E);
    float* w = vector(&m->out_norm);
    or_rmsnorm_rows(x + (int64_t)first * E, n, E, w, m->c.rms_eps, xn);
    matmul(m, &m->output, xn, n, logits);
    if (m->c.logit_scale != 0.0f) {
        float inv = 1.0f / m->c.logit_scale;
        for (int64_t i = 0; i < (int64_t)n * m->output.rows; i++) logits[i] *= inv;
    }
    free(w); free(xn);
}

/* LayerStream.EmbedRow (LayerStream.cs:235-254), scaled like Transformer.cs:93-94. */
static int embed(or_model* m, const int32_t* tokens, int T, float* x, char* err, int errlen)
{
    int E = m->c.embd;
    for (int t = 0; t < T; t++) {
        if (tokens[t] < 0 || tokens[t] >= m->embd.rows) { seterr(err, errlen, "Token id is outside the vocabulary."); return -1; }
        or_decode_row(m->embd.type, m->embd.data + (int64_t)tokens[t] * m->embd.row_bytes, E, x + (int64_t)t * E);
    }
    if (m->c.embedding_scale != 0.0f) for (int64_t i = 0; i < (int64_t)T * E; i++) x[i] *= m->c.embedding_scale;
    return 0;
}

int or_forward(or_model* m, or_seq* sq, const int32_t* tokens, int T, int pos0, int all_logits, float* out, char* err, int errlen)
{
    if (!sq) sq = m->own;
    if (T == 0) { seterr(err, errlen, "No tokens to run."); return -1; }
    if (pos0 > sq->length) { seterr(err, errlen, "pos0 is past the cached positions."); return -1; }
    if (pos0 + T > m->max_context) { seterr(err, errlen, "The prompt and reply need more positions than the context."); return -1; }
    sq->length = pos0;
    reserve(m, sq, pos0 + T);
    float* x = (float*)malloc(sizeof(float) * (size_t)T * m->c.embd);
    if (embed(m, tokens, T, x, err, errlen)) { free(x); return -1; }
    m->each_token = 0;
    for (int l = 0; l < m->c.layers; l++) layer(m, l, x, T, pos0, sq, NULL);
    head(m, x, T, all_logits ? 0 : T - 1, out);
    sq->length = pos0 + T;
    free(x);
    return 0;
}

int or_forward_batch(or_model* m, or_seq* const* seqs, const int32_t* tokens, int N, float* out, char* err, int errlen)
{
    if (N == 0) { seterr(err, errlen, "ForwardBatch needs one token for each sequence."); return -1; }
    batch_rows br;
    br.seq = (or_seq**)malloc(sizeof(or_seq*) * (size_t)N);
    br.pos = (int*)malloc(sizeof(int) * (size_t)N);
    br.maxn = 0;
    for (int i = 0; i < N; i++) {
        or_seq* sq = seqs[i];
        for (int j = 0; j < i; j++) if (seqs[j] == sq) { seterr(err, errlen, "A sequence can take one token per batch step."); free(br.seq); free(br.pos); return -1; }
        int pos = sq->length;
        if (pos + 1 > m->max_context) { seterr(err, errlen, "The prompt and reply need more positions than the context."); free(br.seq); free(br.pos); return -1; }
        br.seq[i] = sq; br.pos[i] = pos;
        if (pos + 1 > br.maxn) br.maxn = pos + 1;
        reserve(m, sq, pos + 1);
    }
    float* x = (float*)malloc(sizeof(float) * (size_t)N * m->c.embd);
    if (embed(m, tokens, N, x, err, errlen)) { free(x); free(br.seq); free(br.pos); return -1; }
    m->each_token = 1;
    for (int l = 0; l < m->c.layers; l++) layer(m, l, x, N, 0, NULL, &br);
    head(m, x, N, 0, out);
    m->each_token = 0;
    for (int i = 0; i < N; i++) seqs[i]->length = br.pos[i] + 1;
    free(x); free(br.seq); free(br.pos);
    return 0;
}

int or_layer(or_model* m, int l, float* x, int T, int pos0, or_seq* sq, char* err, int errlen)
{
    if (!sq) sq = m->own;
    if (l < 0 || l >= m->c.layers) { seterr(err, errlen, "bad layer"); return -1; }
    reserve(m, sq, pos0 + T);
    m->each_token = 0;
    layer(m, l, x, T, pos0, sq, NULL);
    return 0;
}

/* Sampler.Sample greedy (Engine.cs:356-360): strict '>' keeps the lowest index on ties. */
int or_argmax(const float* logits, int n)
{
    int best = 0;
    for (int i = 1; i < n; i++) if (logits[i] > logits[best]) best = i;
    return best;
}

/* Sampler.Sample (Engine.cs:361-380) with the generator's uniform draw passed in (rng.NextDouble(), read only at
 * temperature > 0). The sums run one term at a time in the reference's order. Array.Sort(keys, idx) on keys -p is an
 * unstable introsort whose order among equal probabilities is the .NET runtime's own; this restatement orders them
 * by ascending id (a total order: p descending, then id ascending), the order the device's stable radix sort gives.
 * *margin (optional) = the distance, relative to sum(p), from the draw's running remainder (and, for top_p < 1, from
 * the nucleus limit) to the nearest boundary between two ids around the choice: the choice is the same under any
 * summation order whose rounding error stays below it (the boundary before the first id is an exact zero and does
 * not count). 0 when the choice fell back (no prefix reached the target). */
typedef struct { double p; int id; } or_samp_item;

static int or_samp_cmp(const void* a, const void* b)
{
    const or_samp_item* x = (const or_samp_item*)a;
    const or_samp_item* y = (const or_samp_item*)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return (x->id > y->id) - (x->id < y->id);
}

int or_sample(const float* logits, int n, double temperature, double top_p, double draw, double* margin)
{
    int best = or_argmax(logits, n);
    if (margin) *margin = 1.0;
    if (temperature <= 0) return best;
    float max = logits[best];
    double* p = (double*)malloc(sizeof(double) * (size_t)n);
    double sum = 0;
    for (int i = 0; i < n; i++) {
        float d = logits[i] - max;
        p[i] = exp((double)d / temperature);
        sum += p[i];
    }
    int out = -1;
    double m = 0;
    if (top_p >= 1.0) {
        double r = draw * sum;
        for (int i = 0; i < n; i++) {
            double before = r;
            r -= p[i];
            if (r <= 0) { out = i; m = (i == 0 ? -r : fmin(before, -r)) / sum; break; }
        }
        if (out < 0) out = best;
    } else {
        or_samp_item* it = (or_samp_item*)malloc(sizeof(or_samp_item) * (size_t)n);
        for (int i = 0; i < n; i++) { it[i].p = p[i]; it[i].id = i; }
        qsort(it, (size_t)n, sizeof(or_samp_item), or_samp_cmp);
        double cum = 0, limit = top_p * sum, mn = 0;
        int k = 0;
        while (k < n) {
            double before = cum;
            cum += it[k].p;
            k++;
            if (cum >= limit) { mn = (k == 1 ? cum - limit : fmin(limit - before, cum - limit)) / sum; break; }
        }
        double pick = draw * cum;
        for (int i = 0; i < k; i++) {
            double before = pick;
            pick -= it[i].p;
            if (pick <= 0) { out = it[i].id; m = fmin((i == 0 ? -pick : fmin(before, -pick)) / sum, mn); break; }
        }
        if (out < 0) out = it[0].id;
        free(it);
    }
    free(p);
    if (margin) *margin = m;
    return out;
}
