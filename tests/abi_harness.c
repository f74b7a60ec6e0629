/* A host with no Python: replays, through the C ABI alone, the calls LayeredBackend.Generate makes on its
 * Transformer for a greedy reply (src/Engine.cs:135-250), the sequence a C# host bound by P/Invoke would make.
 *
 *   1. the reply decoded token by token: Forward of the prompt, then Forward([id]) per token, Sampler's greedy argmax
 *      on the host (src/Engine.cs:356-360);
 *   2. the same reply with guess-ahead (src/Engine.cs:196-231, Guess :311-327): a prompt-lookup draft checked in one
 *      all-logits Forward, the agreeing guesses kept, Truncate past them;
 *   3. a second turn that shares the first turn's prefix: Truncate to the common prefix, Forward of the rest
 *      (src/Engine.cs:144-149), against a fresh sequence that runs the whole conversation (logits within 2e-2);
 *   4. the reply from wl_generate_greedy (ids chained on the device) and from wl_forward_argmax.
 *
 * Guesses are capped at 7 so that a checking pass has at most 8 rows: such rows run on the per-column matvec, bit for
 * bit a single-token pass, so guess-ahead cannot change a token here (the reference's assumption, Engine.cs:157).
 * Prints "ok" and exits 0 when all replies agree; any failure prints the call and wl_last_error() and exits 1.
 *
 *   gcc -O2 -I include tests/abi_harness.c -L windlass_b200 -lwindlass_cuda -Wl,-rpath,$PWD/windlass_b200
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "windlass.h"

#define PROMPT 32
#define REPLY 40
#define MAX_GUESSES 7

static wl_model* model;
static int vocab;

static void check(int32_t st, const char* what)
{
    if (st == WL_OK) return;
    fprintf(stderr, "%s failed: [%d] %s\n", what, st, wl_last_error());
    exit(1);
}

static int argmax(const float* x, int n)
{
    int best = 0;
    for (int i = 1; i < n; i++) if (x[i] > x[best]) best = i;
    return best;
}

/* Prompt-lookup guessing (Engine.Guess): the latest earlier place where the last 3, 2 or 1 tokens appeared. */
static int guess(const int* h, int n, int max, int* out)
{
    for (int len = n - 1 < 3 ? n - 1 : 3; len >= 1; len--)
        for (int start = n - len - 1; start >= 0; start--) {
            int k = 0;
            while (k < len && h[start + k] == h[n - len + k]) k++;
            if (k < len) continue;
            int from = start + len, count = n - from < max ? n - from : max;
            if (count <= 0) continue;
            memcpy(out, h + from, sizeof(int) * (size_t)count);
            return count;
        }
    return 0;
}

static void plain_reply(const int* prompt, int* reply)
{
    float* logits = malloc(sizeof(float) * (size_t)vocab);
    check(wl_truncate(model, 0), "wl_truncate");
    check(wl_forward(model, NULL, prompt, PROMPT, 0, 0, logits, NULL, NULL, NULL), "wl_forward (prompt)");
    int id = argmax(logits, vocab);
    for (int i = 0; i < REPLY; i++) {
        reply[i] = id;
        check(wl_forward(model, NULL, &id, 1, PROMPT + i, 0, logits, NULL, NULL, NULL), "wl_forward (token)");
        id = argmax(logits, vocab);
    }
    free(logits);
}

static int guessing_reply(const int* prompt, int* reply)
{
    float* all = malloc(sizeof(float) * (size_t)vocab * (MAX_GUESSES + 1));
    int history[PROMPT + REPLY + MAX_GUESSES + 1], hn = PROMPT, produced = 0, cached = PROMPT, kept = 0;
    memcpy(history, prompt, sizeof(int) * PROMPT);
    check(wl_truncate(model, 0), "wl_truncate");
    check(wl_forward(model, NULL, prompt, PROMPT, 0, 0, all, NULL, NULL, NULL), "wl_forward (prompt)");
    int id = argmax(all, vocab);
    while (produced < REPLY) {
        reply[produced++] = id;
        history[hn++] = id;
        if (produced >= REPLY) break;
        int room = REPLY - produced < MAX_GUESSES ? REPLY - produced : MAX_GUESSES;
        int batch[MAX_GUESSES + 1];
        int nd = guess(history, hn, room, batch + 1);
        batch[0] = id;
        if (nd == 0) {
            check(wl_forward(model, NULL, &id, 1, cached, 0, all, NULL, NULL, NULL), "wl_forward (token)");
            cached++;
            id = argmax(all, vocab);
            continue;
        }
        check(wl_forward(model, NULL, batch, nd + 1, cached, 1, all, NULL, NULL, NULL), "wl_forward (check guesses)");
        int m = 0;
        while (m < nd && argmax(all + (size_t)m * vocab, vocab) == batch[1 + m]) m++;
        check(wl_truncate(model, cached + 1 + m), "wl_truncate (past the kept guesses)");
        cached += 1 + m;
        kept += m;
        int next = argmax(all + (size_t)m * vocab, vocab);
        for (int j = 0; j < m && produced < REPLY; j++) {
            reply[produced++] = batch[1 + j];
            history[hn++] = batch[1 + j];
        }
        id = next;
    }
    free(all);
    return kept;
}

int main(void)
{
    wl_options o;
    wl_options_init(&o);
    o.max_context = 256;
    wl_synth_spec s;
    memset(&s, 0, sizeof s);
    strcpy(s.arch, "llama");               /* configs[0] */
    s.layers = 4; s.embd = 512; s.heads = 8; s.kv_heads = 8; s.head_dim = 64; s.ff = 1408; s.vocab = 4096;
    s.context_length = 4096; s.rope_base = 10000.f; s.rms_eps = 1e-5f; s.sigma = 0.02f;
    s.type_attn = WL_TYPE_Q4_K; s.type_attn_v = WL_TYPE_Q4_K; s.type_ffn = WL_TYPE_Q4_K;
    s.type_ffn_down = WL_TYPE_Q8_0; s.type_embd = WL_TYPE_Q6_K; s.type_output = WL_TYPE_Q6_K;
    check(wl_open_synthetic(&s, &o, &model), "wl_open_synthetic");
    wl_info info;
    check(wl_info_get(model, &info), "wl_info_get");
    vocab = info.vocab;

    int prompt[PROMPT], a[REPLY], b[REPLY], c[REPLY];
    unsigned x = 12345u;
    for (int i = 0; i < PROMPT; i++) { x = x * 1103515245u + 12345u; prompt[i] = (int)((x >> 8) % (unsigned)vocab); }
    plain_reply(prompt, a);
    int kept = guessing_reply(prompt, b);
    if (memcmp(a, b, sizeof a) != 0) { fprintf(stderr, "guess-ahead changed the reply\n"); return 1; }

    /* device greedy: the first id from wl_forward_argmax, the rest chained on the device */
    check(wl_truncate(model, 0), "wl_truncate");
    int32_t first, n = 0;
    check(wl_forward_argmax(model, NULL, prompt, PROMPT, 0, 0, &first, NULL, NULL, NULL), "wl_forward_argmax");
    c[0] = first;
    check(wl_generate_greedy(model, NULL, first, REPLY - 1, NULL, 0, 8, c + 1, &n, NULL), "wl_generate_greedy");
    if (n != REPLY - 1 || memcmp(a, c, sizeof a) != 0) { fprintf(stderr, "device greedy differs\n"); return 1; }

    /* a second turn over the first turn's prefix, against a fresh sequence running the whole conversation */
    int conv[PROMPT + REPLY + 8];
    memcpy(conv, prompt, sizeof prompt);
    memcpy(conv + PROMPT, a, sizeof a);
    for (int i = 0; i < 8; i++) conv[PROMPT + REPLY + i] = (i * 577 + 3) % vocab;
    const int total = PROMPT + REPLY + 8, common = PROMPT + REPLY - 1;
    float* l1 = malloc(sizeof(float) * (size_t)vocab);
    float* l2 = malloc(sizeof(float) * (size_t)vocab);
    check(wl_truncate(model, common), "wl_truncate (common prefix)");
    check(wl_forward(model, NULL, conv + common, total - common, common, 0, l1, NULL, NULL, NULL), "wl_forward (turn 2)");
    wl_seq* fresh;
    check(wl_seq_new(model, &fresh), "wl_seq_new");
    check(wl_forward(model, fresh, conv, total, 0, 0, l2, NULL, NULL, NULL), "wl_forward (whole conversation)");
    int32_t len = 0;
    check(wl_seq_length(fresh, &len), "wl_seq_length");
    /* the fresh pass runs the whole conversation on the tensor-core GEMM, the second turn's prefix came token by token:
     * equal within the stated tolerance of tensor-core prefill logits (2e-2 max-abs) */
    float md = 0.f;
    for (int i = 0; i < vocab; i++) { const float d = l1[i] > l2[i] ? l1[i] - l2[i] : l2[i] - l1[i]; if (d > md) md = d; }
    if (len != total || !(md <= 2e-2f)) { fprintf(stderr, "second turn differs: max |d| %g\n", md); return 1; }
    check(wl_seq_free(fresh), "wl_seq_free");
    free(l1);
    free(l2);

    wl_stats st;
    check(wl_stats_get(model, &st), "wl_stats_get");
    check(wl_close(model), "wl_close");
    printf("ok: %d tokens, %d guesses kept, %lld forward calls, %lld kernel launches\n", REPLY, kept,
           (long long)st.forward_calls, (long long)st.kernel_launches);
    return 0;
}
