// Launch wrappers of the device kernels (all defined in wl_kernels.cu). Every wrapper enqueues on `stream` and
// returns without synchronising; shapes are checked by the callers (wl_model.cpp, wl_api.cpp).
#pragma once
#include <climits>
#include <cstdint>
#include <cuda_runtime.h>

namespace wl {

// Where row t of a step keeps its fp16 KV cache: layer l's keys start at k + l*layer_stride (values likewise at
// v + l*layer_stride), position p at + p*kv_dim.
struct RowKV {
    uint16_t* k;
    uint16_t* v;
    int64_t layer_stride;
};

namespace k {

// ---- the tensor-parallel all-reduce fused into the matvec that produces it and the norm that consumes it ----
// Every rank holds one buffer, mapped into every peer's process. The producer of a partial pushes each of its output
// values into every rank's buffer (its own included) as an 8-byte element {value bits, flag}, the flag derived from
// the all-reduce's sequence number q; an element is written by one 8-byte store, so a reader that sees the flag also
// sees the value, and neither side needs a fence, a separate announcement or a read over NVLink. The consuming norm
// polls its own buffer (bounded in time) until every rank's elements of its rows carry q's flag, then sums the ranks'
// values in rank order, so every rank gets bit-identical sums. The Q4_K decode matvec stores the elements from its
// epilogue (ArOut); any other producer writes its partial into this rank's staging slot and ar_push sends it.
// Sequence numbers are epoch * AR_STEP + index within the step; the epoch is a device counter the step's embedding
// kernel advances, so graph replays need no host input, and the slot (the index mod AR_SLOTS) is known when the step
// is enqueued. A rank writes slot q % AR_SLOTS of a peer only after its own all-reduce q - 1 has received the peer's
// q - 1 values, which the peer produced after its consumer of q - 2 had finished: two slots would do, four are kept.
// Layout: header (the epoch u64 at AR_EPOCH), staging [AR_SLOTS][AR_COLS][E] f32, then the pushed elements
// [AR_SLOTS][AR_MAX_RANKS source][AR_COLS][E] u64. The buffer starts zeroed: flags always have the top bit set.
constexpr int AR_SLOTS = 4;
constexpr int AR_MAX_RANKS = 8;
constexpr int AR_STEP = 1024;                   // most fused all-reduces in one step (a multiple of AR_SLOTS)
constexpr int AR_COLS = 8;                      // columns (decode rows) one slot holds
constexpr size_t AR_HEADER = 1024;              // the epoch u64 at AR_EPOCH
constexpr size_t AR_EPOCH = 512;
static_assert(AR_STEP % AR_SLOTS == 0, "the slot of an all-reduce must not depend on the epoch");
inline size_t ar_slot_offset(int idx, int E) { return AR_HEADER + (size_t)(idx % AR_SLOTS) * AR_COLS * E * sizeof(float); }
inline size_t ar_ll_offset(int E) { return AR_HEADER + (size_t)AR_SLOTS * AR_COLS * E * sizeof(float); }
inline size_t ar_buffer_bytes(int E)
{
    return ar_ll_offset(E) + (size_t)AR_SLOTS * AR_MAX_RANKS * AR_COLS * E * sizeof(unsigned long long);
}
// The producer's side: every rank's pushed-element region (peers' mapped into this process) and this rank's epoch.
struct ArOut {
    unsigned long long* ll[AR_MAX_RANKS];
    const unsigned long long* epoch;
    int idx, G, rank, E;
};
// The consumer's side: this rank's pushed-element region.
struct ArIn {
    const unsigned long long* ll;
    const unsigned long long* epoch;            // this rank's step counter
    int* err;                                   // set to 2 when a wait gives up
    int idx, G, rank, E, row0;                  // row0: first partial row the consumer's row 0 reads
    long long wait_ns;                          // how long a wait for a peer may last before it gives up
};
constexpr long long AR_WAIT_NS = 10000000000LL; // 10 s: far beyond any skew between ranks that are running
// Pushes T rows of E floats (src, row-major) into every rank's elements of all-reduce ao.idx, source ao.rank.
void ar_push(const float* src, int T, const ArOut& ao, cudaStream_t s);
// Runs the fused all-reduce's consumer on this GPU against a peer that never pushes (elements nothing writes), with
// its wait limited to wait_ns: returns the error code the kernel recorded (2 when the wait gave up, as it must).
int selftest_ar_wait(long long wait_ns);

// Copies the I-quant tables into the current device's constant memory (once per device).
void init_tables();
// Kernels launched by this process so far; note_launch() checks and counts a launch made in another file.
int64_t launches();
void note_launch();
// Takes back n counted launches that were captured into a graph rather than run.
void uncount_launches(int64_t n);

// Quants.DecodeRow for n consecutive values (n a multiple of the block size), bit-exact.
void dequant(int type, const void* blocks, int64_t n, float* out, cudaStream_t s);
// Rows `tokens[t]` of an embedding matrix (cols values each, row_bytes apart) decoded to x[t*cols...], times scale
// when scale != 0 (LayerStream.EmbedRow + Transformer.cs:93-94). Out-of-range ids set *bad_token.
void embed(int type, const uint8_t* w, int64_t row_bytes, int rows, int cols, const int32_t* tokens, int T,
           float scale, float* x, int32_t* bad_token, cudaStream_t s, unsigned long long* epoch = nullptr);

// y[t*ldy + r] = W[r] . x[t*ldx...] for t < ncols (1..8), rows r of W (row_bytes apart). Each column is computed
// with the same instruction sequence whatever ncols is, so a column's result does not depend on its neighbours.
void matvec(int type, const uint8_t* w, int64_t row_bytes, int rows, int cols, const float* x, int64_t ldx,
            int ncols, float* y, int64_t ldy, cudaStream_t s);

// Activations prepared for the tensor-core matvec: per column and 256-value superblock one XP_COL-byte block of three
// signed 8-bit digit planes (pitch XP_DIGIT) of the values under a power-of-two unit, and at XP_REC the f16 hi/lo
// sums of every 32 values and the unit.
constexpr int XP_DIGIT = 288, XP_REC = 864, XP_COL = 992;
constexpr size_t xprep_bytes_c(int cols, int nc) { return (size_t)nc * (size_t)(cols / 256) * XP_COL + 256; }
struct XPrep {
    uint8_t* blocks;    // [nc][cols/256][XP_COL]
    int cols = 0, nc = 0;
};
size_t xprep_bytes(int cols, int nc);
XPrep xprep_view(void* scratch, int cols, int nc);
// The static scratch of wl_matvec_static: a 256-byte error word slot, then xprep_bytes(STATIC_MAX_COLS, 8).
constexpr int STATIC_MAX_COLS = 32768;
constexpr size_t STATIC_SCRATCH_BYTES = 256 + xprep_bytes_c(STATIC_MAX_COLS, 8);
// Device address of this device's static scratch (looked up once per device with cudaGetSymbolAddress).
void* static_scratch();
// x[t*ldx + i] for t < nc (1..8), cols a multiple of 256.
void xprep(const float* x, int64_t ldx, int cols, int nc, const XPrep& p, cudaStream_t s);
// x[t] += o[t] * rs (when o), then y[t] = RmsNormRows(x[t]) * w for T rows of E values, and when p is given y's
// activations prepared as xprep would (bit-identical), in one kernel. E a multiple of 256, at most 8192.
bool norm_prep_supported(int E);
// With ar, o is the rank-ordered sum of every rank's partial in the fused all-reduce's slot instead (o unused).
// With moe, o is the mixture-of-experts combine of each row's K chosen experts (moe_combine's arithmetic, o unused).
struct MoeIn {
    const float* y = nullptr;       // [T*K][E] the chosen experts' outputs, pair t*K + j
    const int32_t* sel = nullptr;   // [T*K] expert ids
    const float* wts = nullptr;     // [T*K] weights
    int K = 0;
};
void norm_prep(float* x, const float* o, float rs, int T, int E, const float* w, float eps, float* y, const XPrep* p,
               cudaStream_t s, const ArIn* ar = nullptr, const MoeIn* moe = nullptr);
// A TMA tensor map over a weight matrix (CUtensorMap, 128 bytes, 64-byte aligned), made once per matrix.
struct alignas(64) WeightMap {
    uint8_t bytes[128];
    bool valid = false;
};
// True when `type` has a tensor-core matvec and the weights' alignment allows it.
bool mma_supported(int type, const uint8_t* w, int64_t row_bytes, int cols);
// Map over rows_total rows (all experts of a stacked tensor); boxes of one superblock x 32 rows.
void make_weight_map(int type, const uint8_t* w, int64_t rows_total, int64_t row_bytes, WeightMap* out);
// y[t*ldy + r] = W[row_base + r] . x[t] for r < rows, from prepared activations (same contract as matvec). A stuck
// copy sets *err (device memory) instead of hanging.
void matvec_mma(int type, const WeightMap& map, int row_base, int rows, int cols, const XPrep& p, float* y,
                int64_t ldy, int* err, cudaStream_t s);
// Sets the shared-memory attribute of every column count's matvec_mma kernel on the current device (once per device;
// later calls return at once), so that no later matvec_mma call has a first-use step.
void prepare_matvec_mma();

// Q4_K and Q6_K on the tensor cores from tile-major weights: each 16-row x one-superblock tile contiguous and laid
// out for the kernel's fragment reads (made once by make_tiles, tile_bytes bytes, 16-byte aligned); then
// y[t*ldy + r] = W[row_base + r] . x[t] from prepared activations (same contract as matvec), row_base a multiple of 16.
constexpr int Q6K_TILE = 3360;     // bytes of one Q6_K tile: 16 rows x one 210-byte superblock
bool tiles_supported(int type, int cols);
// Q8_0, IQ4_XS and IQ2_XXS (type 8, 23, 16) in the same scheme (wl_mmv_i8.cu): tiles of 16 rows x 256 values, an
// integer tensor-core matvec over the values decoded to int8; tiles_supported, tile_bytes, make_tiles and matvec_tiles
// cover them too.
bool i8_tiles_supported(int type, int cols);
int64_t i8_tile_bytes(int type, int rows, int cols);
void make_i8_tiles(int type, const uint8_t* w, int rows, int cols, int64_t row_bytes, uint8_t* tiles, cudaStream_t s);
void matvec_i8_tiles(int type, const uint8_t* tiles, int rows, int cols, const XPrep& p, float* y, int64_t ldy, int* err,
                     cudaStream_t s);
void init_i8_tables();
int64_t tile_bytes(int type, int rows, int cols);
void make_tiles(int type, const uint8_t* w, int rows, int cols, int64_t row_bytes, uint8_t* tiles, cudaStream_t s);
// With ao (Q4_K only) the outputs are not written to y but pushed as all-reduce ao.idx's elements.
void matvec_tiles(int type, const uint8_t* tiles, int row_base, int rows, int cols, const XPrep& p, float* y,
                  int64_t ldy, int* err, cudaStream_t s, const ArOut* ao = nullptr);

// Two Q4_K matrices with the same columns and activations (q and k, gate and up) in one tensor-core matvec launch:
// y_a[t*ldy_a + r] = A[row_base_a + r] . x[t], y_b likewise; each row's result is the one matvec_tiles gives.
void matvec_tiles2(const uint8_t* tiles_a, int row_base_a, int rows_a, float* y_a, int64_t ldy_a, const uint8_t* tiles_b,
                   int row_base_b, int rows_b, float* y_b, int64_t ldy_b, int cols, const XPrep& p, int* err,
                   cudaStream_t s);

// The mixture-of-experts grouped matvec (Q4_K experts, one activation column per pair): for every pair i < npairs
// (token i / K and its expert sel[i], read on the device), y[i*ldy + r] = E_sel[i][r] . x[col] for the expert's
// expert_rows rows (expert e's rows start at row_base + e * expert_rows of the tiles), col = i / K when x_per_token
// else i. Each pair's result is the one a matvec of that expert alone gives. Under tensor parallelism the tiles hold
// experts e_lo .. e_lo + e_n - 1 only (local expert e - e_lo at row_base + (e - e_lo) * expert_rows), and the pairs of
// other experts are skipped: their outputs are not written.
void matvec_pairs(const uint8_t* tiles, int row_base, int expert_rows, int cols, const int32_t* sel, int npairs, int K,
                  bool x_per_token, const XPrep& p, float* y, int64_t ldy, int* err, cudaStream_t s, int e_lo = 0,
                  int e_n = INT_MAX);
// Gate and up of every pair in one launch: matvec_pairs of A into ya and of B (same shape, stacked the same way) into
// yb, activations per token (x_per_token), each CTA's result what matvec_pairs gives.
void matvec_pairs2(const uint8_t* tiles_a, const uint8_t* tiles_b, int expert_rows, int cols, const int32_t* sel,
                   int npairs, int K, const XPrep& p, float* ya, float* yb, int64_t ldy, int* err, cudaStream_t s,
                   int e_lo = 0, int e_n = INT_MAX);
// MoeFfn's weighted sum (src/Transformer.cs:289-293) from the pairs' outputs: out[t] = sum over token t's K experts in
// ascending expert order of wts[t*K+j] * y[(t*K+j)*E ...], each step a separately rounded multiply and add from 0.
// Under tensor parallelism only the experts e_lo .. e_lo + e_n - 1 this GPU holds are added (the ranks' sums are
// then all-reduced).
void moe_combine(const float* y, const int32_t* sel, const float* wts, int T, int K, int E, float* out, cudaStream_t s,
                 int e_lo = 0, int e_n = INT_MAX);
// Adds to *count the number of distinct experts among sel[0 .. n) (Transformer.ExpertRuns, src/Transformer.cs:287).
void count_experts(const int32_t* sel, int n, unsigned long long* count, cudaStream_t s);

// Q4_K GEMM on the tcgen05 tensor cores for T > 8 activation rows (prefill, large batches): y[t*ldy + r] =
// W[row_base + r] . x[t*ldx ...] from the tile-major weights, with fp32-level accuracy (bf16 hi/lo planes of both
// operands, three MMAs per slice, fp32 accumulation in tensor memory). scratch holds gemm_scratch_bytes(T, cols) bytes
// (the activations' bf16 planes); a stuck wait sets *err.
bool gemm_supported(int type, int cols);
// Fewer rows than this go through the integer tensor-core matvec in 8-column launches instead: the GEMM's time hardly
// depends on T up to its 128-token tile (8192 x 8192 Q4_K: about 200 us at 16 or 64 tokens), against about 19 us a
// chunk of eight for the matvec (measured on B200: crossing near 88 rows for Q4_K, 60 for Q6_K).
int gemm_min_rows(int type);
size_t gemm_scratch_bytes(int T, int cols);
void gemm_tiles(int type, const uint8_t* tiles, int row_base, int rows, int cols, const float* x, int64_t ldx, int T,
                float* y, int64_t ldy, void* scratch, int* err, cudaStream_t s);

// RmsNormRows (Transformer.cs:454-464): n rows of dim values; y may alias x.
void rmsnorm(const float* x, int n, int dim, const float* w, float eps, float* y, cudaStream_t s);
// y[t*n + i] += b[i] for T rows (AddBias, Transformer.cs:442-451).
void add_bias(float* y, const float* b, int T, int n, cudaStream_t s);
// Rope (Transformer.cs:418-433) on T rows of `heads` heads; positions pos[t]; table[pos*rope_dims + 2i (+1)] = cos, sin.
void rope(float* x, int T, int heads, int head_dim, int rope_dims, int neox, const int32_t* pos, const float* table,
          cudaStream_t s);
// K/V rows t (kd values) to fp16 at position pos[t] of layer `layer` of row t's cache (ToHalf,
// Transformer.cs:342-348).
void kv_append(const float* k, const float* v, int T, int kd, const RowKV* rows, int layer, const int32_t* pos,
               cudaStream_t s);
// Attention (Transformer.cs:351-395): row t, head h attends to positions 0..pos[t] of its own cache. part is a
// workspace of attention_part_floats(heads, kv_heads, head_dim) floats for the split-range partials. For up to
// ATT_PART_ROWS rows each row's positions are split into S ranges, S fixed by the model's KV-head count (16 at 8 or
// more KV heads, up to 64 at one, so that S x kv_heads CTAs cover the SMs): a row's result never depends on the
// other rows; with prep (T <= 8) the output is also written as prepared activations, and the call
// returns whether it did.
constexpr int ATT_PART_ROWS = 64;
constexpr int ATT_SPLITS = 16;                  // S at 8 or more KV heads
constexpr int ATT_MAX_SPLITS = 64;
inline int attention_splits_for(int kv_heads)
{
    const int s = 128 / (kv_heads > 0 ? kv_heads : 1);
    return s < ATT_SPLITS ? ATT_SPLITS : s > ATT_MAX_SPLITS ? ATT_MAX_SPLITS : s;
}
// The partials, their (max, sum) pairs, then one ticket counter per (row, KV head); the counters must be zero when the
// workspace is first used (each merging CTA resets its counter for the next launch).
inline size_t attention_part_floats(int heads, int kv_heads, int head_dim)
{
    return (size_t)ATT_PART_ROWS * attention_splits_for(kv_heads) * heads * (head_dim + 2) +
           (size_t)ATT_PART_ROWS * kv_heads;
}
int attention_splits(int T, int kv_heads);
bool attention_supported(int heads, int kv_heads, int head_dim);
// RoPE and the KV append of a one-row decode step done inside the attention, in place of rope_append (same
// arithmetic, same bits): q is read unrotated and rotated as it is staged; the CTA whose position range holds the
// row's new position pos[0] rotates k and writes k and v there, in the cache and in its staged tile. No other CTA
// reads that position, so nothing waits for the append.
struct AttnRope {
    const float* k = nullptr;       // [KV heads * head_dim], unrotated
    const float* v = nullptr;
    const float* table = nullptr;   // the rope table (cos, sin per position and pair)
    int rope_dims = 0, neox = 0;
};
bool attention(const float* q, int T, int heads, int kv_heads, int head_dim, float scale, const RowKV* rows,
               int layer, const int32_t* pos, float* part, float* out, const XPrep* prep, cudaStream_t s,
               const AttnRope* rope = nullptr);
// RoPE on q (heads) and k (kv heads) of T rows, then k and v appended to the fp16 caches at pos[t] (Rope,
// Transformer.cs:418-433, and ToHalf, :342-348), in one kernel; k is left unrotated in its buffer.
void rope_append(float* q, const float* k, const float* v, int T, int heads, int kv_heads, int head_dim, int rope_dims,
                 int neox, const int32_t* pos, const float* table, const RowKV* rows, int layer, cudaStream_t s);
// Per-head QK-norm then rope_append in one kernel, bit for bit the two rmsnorm passes and rope_append; false (nothing
// launched) unless the rope is NEOX over the whole head and head_dim is 64, 128 or 256.
bool qknorm_rope_append(float* q, const float* k, const float* v, int T, int heads, int kv_heads, int head_dim,
                        int rope_dims, int neox, const float* qw, const float* kw, float eps, const int32_t* pos,
                        const float* table, const RowKV* rows, int layer, cudaStream_t s);
// SwiGlu into g (as swiglu) for T rows of F values, and g's prepared activations (F a multiple of 256, T <= 8).
void swiglu_prep(float* g, const float* u, int T, int F, const XPrep& p, cudaStream_t s);
// g[i] = g[i]/(1+exp(-g[i])) * u[i] (SwiGlu, Transformer.cs:247).
void swiglu(float* g, const float* u, int64_t n, cudaStream_t s);
// x[i] += o[i] * rs (Transformer.cs:225,231).
void residual(float* x, const float* o, float rs, int64_t n, cudaStream_t s);
// The tensor-parallel head's logits: src is [G][n][vp] (rank g's rows g*vp ..), dst[t*V + v] = src[g][t][v - g*vp].
void vocab_gather(const float* src, int G, int n, int vp, int V, float* dst, cudaStream_t s);
// x[i] *= f.
void scale(float* x, float f, int64_t n, cudaStream_t s);
// Greedy selection on n rows of V logits (Sampler.Sample at temperature 0, Engine.cs:356-360; Argmax, :329-334):
// ids[r] = the lowest index of row r's largest value (0 when x[0] is NaN). key[n] and count[n] are zero before the
// launch and after it. With next_tok set, next_tok[r] = ids[r] and next_pos[r] += 1 (a chained decode step).
void argmax(const float* logits, int V, int n, unsigned long long* key, unsigned* count, int32_t* ids,
            int32_t* next_tok, int32_t* next_pos, cudaStream_t s);
// Blocks per row of that launch (for tests of its arithmetic).
int64_t argmax_blocks(int V, int n);
// Sampler.Sample (src/Engine.cs:361-380) on one row of V device logits with the host's uniform draw in [0, 1) (its
// rng.NextDouble(); unused at temperature <= 0): *out_id (device) = the chosen id. ws is sample_workspace_bytes(V)
// of device memory, its first 256 bytes zeroed once by sample_workspace_init; rows sampled one after another on one
// stream may share it.
size_t sample_workspace_bytes(int V);
void sample_workspace_init(void* ws, cudaStream_t s);
void sample(const float* logits, int V, double temperature, double top_p, double draw, void* ws, int32_t* out_id,
            cudaStream_t s);
// Route (Transformer.cs:315-340) for T rows of n router logits: sel[t*k+j], wts[t*k+j].
// With count_one (T = 1 only), *count_one += k: a single token's picks are k distinct experts, so the step needs no
// count_experts launch.
void route(const float* logits, int T, int n, int k, int renorm, int32_t* sel, float* wts, cudaStream_t s,
           unsigned long long* count_one = nullptr);
// outp[t*E + d] += w * ye[i*E + d] for the gathered rows i of one expert (MoeFfn, Transformer.cs:289-293).
void scatter_add(float* outp, const float* ye, const int32_t* toks, const float* w, int n, int E, cudaStream_t s);
// xe[i*E..] = xn[toks[i]*E..].
void gather_rows(float* xe, const float* xn, const int32_t* toks, int n, int E, cudaStream_t s);
// outp[t*E + d] += f_t * sh[t*E + d], f_t = gl ? 1/(1+exp(-gl[t])) : 1 (shared expert, Transformer.cs:296-309).
void shared_expert_add(float* outp, const float* sh, const float* gl, int T, int E, cudaStream_t s);

// Synthetic weights of wl_synth_tensor / wl_open_synthetic.
// F32 tensors get offset + sigma*z (offset 1 for norm weights); quantized types get sigma*z, quantized.
void synth(int type, uint64_t seed, uint32_t tid, int64_t rows, int64_t cols, float sigma, float offset, uint8_t* out,
           cudaStream_t s);

}  // namespace k
}  // namespace wl
