/* libwindlass_cuda: the C ABI of the B200-native Windlass quantized transformer forward.
 *
 * The reference engine (C#, .NET Framework 4.8) reaches its forward pass only through the Transformer object
 * (src/Transformer.cs) inside LayeredBackend (src/Engine.cs). This library replaces that object: a C# host binds
 * these entry points with P/Invoke and keeps its server, BatchEngine, Playbook,
 * tokenizer and sampler unchanged. Plain pointers and sizes only; no C++ or CUDA types cross the boundary except the
 * opaque `stream` arguments of the kernel-level test exports, which are cudaStream_t values (NULL = default stream).
 *
 * Error convention: every function returns WL_OK (0) or a WL_E* status and never aborts or exits. wl_last_error()
 * returns the calling thread's message for the last failure. Statuses map to the reference's exceptions as noted.
 * Threading: one call at a time per model (the reference serialises on LayeredBackend._run, src/Engine.cs:138 and
 * src/BatchEngine.cs:111). Progress callbacks run on the calling thread between stages.
 */
#ifndef WINDLASS_H
#define WINDLASS_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WL_OK            0
#define WL_EINVAL        1   /* ArgumentException: bad shape, pos0 past the cache, context overflow, bad token id */
#define WL_EUNSUPPORTED  2   /* NotSupportedException: architecture, weight type or layout the engine cannot run */
#define WL_EIO           3   /* IOException: the file cannot be opened or read */
#define WL_EFORMAT       4   /* InvalidDataException: the file is not valid GGUF */
#define WL_ENOMEM        5   /* device or pinned host memory exhausted */
#define WL_ECUDA         6   /* a CUDA call failed */
#define WL_ENCCL         7   /* an NCCL call failed */
#define WL_ETIMEDOUT     8   /* a bounded device-side wait gave up */
#define WL_CANCELLED     9   /* OperationCanceledException: the cancel flag was set between stages */

/* ggml_type numbers of the weight formats (src/Gguf.cs:19-25). */
#define WL_TYPE_F32      0
#define WL_TYPE_F16      1
#define WL_TYPE_Q4_0     2
#define WL_TYPE_Q4_1     3
#define WL_TYPE_Q5_0     6
#define WL_TYPE_Q5_1     7
#define WL_TYPE_Q8_0     8
#define WL_TYPE_Q2_K    10
#define WL_TYPE_Q3_K    11
#define WL_TYPE_Q4_K    12
#define WL_TYPE_Q5_K    13
#define WL_TYPE_Q6_K    14
#define WL_TYPE_IQ2_XXS 16
#define WL_TYPE_IQ2_XS  17
#define WL_TYPE_IQ3_XXS 18
#define WL_TYPE_IQ1_S   19
#define WL_TYPE_IQ4_NL  20
#define WL_TYPE_IQ3_S   21
#define WL_TYPE_IQ2_S   22
#define WL_TYPE_IQ4_XS  23
#define WL_TYPE_IQ1_M   29
#define WL_TYPE_BF16    30

typedef struct wl_model wl_model;
typedef struct wl_seq wl_seq;

/* onStage(done, total) of Transformer.Forward (src/Transformer.cs:102,106): called after each layer and the head. */
typedef void (*wl_progress_fn)(int32_t done, int32_t total, void* user);

typedef struct wl_options {
    int32_t size;            /* sizeof(wl_options), set by wl_options_init */
    int32_t device;          /* CUDA device ordinal */
    int32_t max_context;     /* positions per sequence; 0 = min(model context_length, 8192) (src/Engine.cs:26,62) */
    int32_t max_batch;       /* most rows in one wl_forward_batch (BatchPlan.MaxBatch = 64, src/Batch.cs:40) */
    int32_t resident;        /* 1 or -1: every weight resident in HBM. 0: layers stream from pinned host memory
                                (LayerStream, src/LayerStream.cs): each layer's weights (and the output head's) are
                                copied into one of two device slots on a copy stream while the previous layer
                                computes; the embedding, norms and biases stay resident. Decode steps then run
                                without CUDA graphs, and prefill_path 1 is refused */
    int32_t prefill_path;    /* T > 8 rows: 0 auto (Q4_K on the tcgen05 GEMM, other formats with a tensor-core
                                matvec in 8-column chunks), 1 fp32 CUDA cores, 2 the integer tensor-core matvec in
                                8-column chunks for every format that has one */
    int32_t use_graphs;      /* 1: replay decode steps from captured CUDA graphs */
    int32_t tp_size;         /* tensor parallelism: ranks that share the model, one GPU each (0 or 1 = one GPU).
                                Every rank opens the same model with its own tp_rank and the same tp_id, and then
                                makes the same calls with the same arguments; each call returns the full logits on
                                every rank. Query/key/value, gate/up and the output head are split by rows, the
                                attention output and down projections by columns, with an NCCL all-reduce after each
                                of the latter two (dense models; head and KV-head counts divisible by tp_size). */
    int32_t tp_rank;         /* this caller's rank, 0 .. tp_size-1; or -1: this one wl_model spans all tp_size GPUs
                                (devices device .. device+tp_size-1), one shard and one host thread per GPU inside
                                this process, for hosts that run a single process (tp_id is then not read). Every
                                call runs all shards at once; progress callbacks come on the calling thread */
    int32_t tp_nccl_only;    /* 0: decode-step all-reduces fused into the producing matvec and the consuming norm over
                                NVLink peer memory (CUDA IPC), falling back to NCCL when the GPUs cannot map each
                                other's memory; 1: NCCL all-reduce only */
    int32_t stream_file;     /* with resident = 0 and a model opened from a GGUF file (one GPU): 1 reads each stage
                                from the file at every use (LayerStream.Acquire's reads, src/LayerStream.cs:182-232):
                                8 MB chunks through a ring of four pinned buffers, O_DIRECT where the file system
                                allows it, on a reader thread that overlaps the reads with the copies, so the host
                                holds no copy of the model; 0 lays every stage out once in pinned host memory */
    int32_t reserved[5];
    uint8_t tp_id[128];      /* the group's id: wl_tp_unique_id on one rank, the same bytes passed to every rank */
} wl_options;

typedef struct wl_info {
    int32_t layers, embd, heads, kv_heads, head_dim, vocab, context_length, max_context;
    int32_t expert_count, expert_used, expert_ff, moe;
    int64_t weight_bytes;    /* quantized weight bytes of all layers and the head held by this rank */
    int64_t device_bytes;    /* device memory the model holds now */
    char arch[32];
    int32_t tp_size, tp_rank;
    int32_t tp_fused;        /* 1: decode-step all-reduces run fused over peer memory (else NCCL) */
} wl_info;

typedef struct wl_stats {
    int64_t bytes_h2d;       /* weight bytes copied host->device (LayerStream.BytesRead, src/LayerStream.cs:83) */
    int64_t expert_runs;     /* experts computed (Transformer.ExpertRuns, src/Transformer.cs:27,287) */
    int64_t forward_calls, batch_calls, tokens;
    double  last_forward_ms;
    int64_t kernel_launches; /* kernels this process has launched from the library (all models) */
} wl_stats;

/* Per weight format: matvec/matmul launches, their summed device time (CUDA events around each launch on the
 * model's stream) and the algorithmic bytes they moved (weights + activations in + outputs), since profiling was
 * switched on with wl_profile(model, 1). */
typedef struct wl_profile_entry {
    int64_t launches;
    double  ms;
    double  bytes;
} wl_profile_entry;
/* wl_profile_get kinds beyond the weight formats. */
#define WL_PROFILE_ATTENTION 40   /* attention and its range merge */
#define WL_PROFILE_NORM      41   /* residual + RmsNorm (+ activation prep) */
#define WL_PROFILE_ROPE      42   /* RoPE + KV append */
#define WL_PROFILE_SWIGLU    43   /* SwiGlu (+ activation prep) */
#define WL_PROFILE_XPREP     44   /* stand-alone activation prep of the tensor-core matvecs */
#define WL_PROFILE_ALLREDUCE 45   /* tensor-parallel collectives (bytes: what each rank sends over NVLink) */

/* Synthetic model (benchmarks and full-size tests): a decoder of the given shape whose weights are generated on the
 * device from a counter hash (seed, tensor, element), N(0, sigma) through Irwin-Hall(12), round-to-nearest quantized.
 * The same bytes come out of the CPU generator of the test oracle. No file is read. */
typedef struct wl_synth_spec {
    char arch[16];           /* "llama", "qwen3" (QK-norm) or "qwen3moe" */
    int32_t layers, embd, heads, kv_heads, head_dim, ff, vocab, context_length;
    int32_t experts, experts_used, expert_ff;
    float rope_base, rms_eps, sigma;
    int32_t type_attn, type_attn_v, type_ffn, type_ffn_down, type_embd, type_output;
    uint64_t seed;
} wl_synth_spec;

void        wl_options_init(wl_options* opt);
const char* wl_last_error(void);
const char* wl_version(void);
/* No counterpart in the reference (it runs on one CPU): a fresh id for a tensor-parallel group (ncclGetUniqueId)
 * into id[0..bytes), bytes >= 128. One rank calls it and hands the bytes to the others (wl_options.tp_id). Needs NCCL
 * (libnccl.so.2, loaded on first use); without it the call returns WL_ENCCL. */
int32_t wl_tp_unique_id(uint8_t* id, int32_t bytes);

/* LayeredBackend.Load (src/Engine.cs:55-91): GgufModelFile.Open + ModelConfig.From + LayerStream + Transformer. */
int32_t wl_open(const char* gguf_path, const wl_options* opt, wl_model** out);
int32_t wl_open_synthetic(const wl_synth_spec* spec, const wl_options* opt, wl_model** out);
int32_t wl_close(wl_model* model);
int32_t wl_info_get(const wl_model* model, wl_info* info);
int32_t wl_stats_get(const wl_model* model, wl_stats* stats);

/* Transformer.NewSequence / Sequence.Truncate / Sequence.Length (src/Transformer.cs:60, src/Batch.cs:28).
 * A sequence owns its fp16 KV cache in device memory; free every sequence before its model. */
int32_t wl_seq_new(wl_model* model, wl_seq** out);
int32_t wl_seq_free(wl_seq* seq);
int32_t wl_seq_truncate(wl_seq* seq, int32_t n);
int32_t wl_seq_length(const wl_seq* seq, int32_t* n);

/* Transformer.Truncate / Transformer.Length on the model's own sequence (src/Transformer.cs:28,57). */
int32_t wl_truncate(wl_model* model, int32_t n);
int32_t wl_length(const wl_model* model, int32_t* n);

/* Transformer.Forward (src/Transformer.cs:77-109): runs tokens[0..T) at positions pos0.. of seq (NULL = the model's
 * own). logits_out (host memory) receives T*vocab floats when all_logits != 0, else the last token's vocab floats.
 * cancel (may be NULL) is polled between stages; a cancelled call returns WL_CANCELLED and leaves the sequence
 * length at pos0. */
int32_t wl_forward(wl_model* model, wl_seq* seq, const int32_t* tokens, int32_t T, int32_t pos0, int32_t all_logits,
                   float* logits_out, volatile const int32_t* cancel, wl_progress_fn progress, void* user);

/* Transformer.ForwardBatch (src/Transformer.cs:132-170): one decode step for N sequences; token i is the next token
 * of seqs[i] at position seqs[i]'s length. Row i of logits_out (N*vocab host floats) is bit-identical to what
 * wl_forward(seqs[i], &tokens[i], 1, ...) returns. */
int32_t wl_forward_batch(wl_model* model, wl_seq* const* seqs, const int32_t* tokens, int32_t N, float* logits_out,
                         volatile const int32_t* cancel, wl_progress_fn progress, void* user);

/* One pass over several sequences' new tokens at once: a decode step that new prompts join (continuous batching, the
 * reference's roadmap item "prompts joining a running batch", which its BatchEngine does not do). Sequence seqs[i]
 * takes counts[i] >= 1 tokens at positions length(seqs[i]).. ; tokens holds them sequence after sequence (sum of
 * counts). logits_out (N*vocab host floats) gets each sequence's last row in sequence order, or, when ids_out is not
 * NULL, ids_out[i] gets that row's greedy id instead (logits_out may then be NULL). Each row attends to its own
 * sequence only; a row's result equals that sequence's own wl_forward of the same tokens (bit for bit when the step
 * has at most 8 rows; beyond that the rows run on the tensor-core GEMM, as a prompt does). Cancel and progress as in
 * wl_forward; a cancelled step leaves every sequence's length unchanged. */
int32_t wl_forward_mixed(wl_model* model, wl_seq* const* seqs, const int32_t* counts, int32_t N, const int32_t* tokens,
                         float* logits_out, int32_t* ids_out, volatile const int32_t* cancel, wl_progress_fn progress,
                         void* user);

/* ---- greedy selection on the device (the caller of Forward, src/Engine.cs:135-250, with Sampler.Sample at
 * temperature 0, :356-360, and the guess-ahead check's Argmax, :329-334). Each id is the lowest index of the largest
 * logit (strict > in index order: ties go to the lower id, NaNs never win, and a NaN at index 0 makes the answer 0),
 * the same bits as the host rule applied to the logits the logits-returning call gives. ---- */

/* wl_forward, returning ids instead of logits: ids_out[0] = the last row's argmax (all_rows = 0), or ids_out[t] =
 * row t's for every t < T (all_rows != 0; the guess-ahead check of Engine.cs:207-216). Same arguments, errors,
 * cancel and progress behaviour. */
int32_t wl_forward_argmax(wl_model* model, wl_seq* seq, const int32_t* tokens, int32_t T, int32_t pos0,
                          int32_t all_rows, int32_t* ids_out, volatile const int32_t* cancel, wl_progress_fn progress,
                          void* user);
/* wl_forward_batch, returning ids_out[i] = the argmax of row i. */
int32_t wl_forward_batch_argmax(wl_model* model, wl_seq* const* seqs, const int32_t* tokens, int32_t N,
                                int32_t* ids_out, volatile const int32_t* cancel, wl_progress_fn progress, void* user);

/* ---- sampling on the device (Sampler.Sample, src/Engine.cs:361-380: the decode loop's choice, :187 and :202, and
 * the batching loop's, src/BatchEngine.cs:164-172). The caller keeps the random generator: `draw` is its next uniform double in [0, 1) (Random.NextDouble()),
 * taken only when temperature > 0, as the reference takes one. temperature <= 0 gives the greedy id (the draw is not
 * read). Otherwise p[i] = exp((logit[i] - max) / temperature) in double; top_p >= 1 picks the first id at which the
 * running sum of p in index order reaches draw * sum(p); top_p < 1 orders ids by p descending, keeps the shortest
 * prefix whose running sum reaches top_p * sum(p), and picks the first id of it at which the running sum reaches
 * draw * (the prefix's sum). The sums are tree-ordered prefix sums where the reference adds one term at a time, and
 * equal probabilities keep ascending ids (a stable sort) where the reference's unstable Array.Sort orders them its
 * own way: a choice can differ only when the draw falls within a few units in the last place of the boundary between
 * two ids, or among exactly equal probabilities. ---- */

/* wl_forward returning the last row's sampled id in *id_out (WL_EINVAL for a draw outside [0, 1) at temperature > 0).
 * Same arguments, errors, cancel and progress behaviour otherwise. */
int32_t wl_forward_sample(wl_model* model, wl_seq* seq, const int32_t* tokens, int32_t T, int32_t pos0,
                          double temperature, double top_p, double draw, int32_t* id_out,
                          volatile const int32_t* cancel, wl_progress_fn progress, void* user);
/* wl_forward_batch returning ids_out[i] = row i sampled with temperature[i], top_p[i] and draws[i] (each batch job's
 * own options and generator, src/BatchEngine.cs:164-172). */
int32_t wl_forward_batch_sample(wl_model* model, wl_seq* const* seqs, const int32_t* tokens, int32_t N,
                                const double* temperature, const double* top_p, const double* draws, int32_t* ids_out,
                                volatile const int32_t* cancel, wl_progress_fn progress, void* user);

/* Greedy decode of seq (NULL = the model's own) chained on the device, the decode loop of Engine.cs:187-203 at
 * temperature 0: step s forwards `token` (s = 0) or ids_out[s-1] at the sequence's next position and writes the
 * argmax of its logits to ids_out[s]. The id never visits the host between steps: `chunk` steps (0 = 16, at most 64)
 * run back to back before their ids are read. Ends after the first id found in stop_ids[0..n_stop) (kept as the last
 * id) or after max_new steps; *n_out = the ids written, and the sequence grows by *n_out (every step forwarded one
 * token). cancel is read before each chunk; a cancelled call returns WL_CANCELLED with *n_out and the sequence at
 * the steps completed. */
int32_t wl_generate_greedy(wl_model* model, wl_seq* seq, int32_t token, int32_t max_new, const int32_t* stop_ids,
                           int32_t n_stop, int32_t chunk, int32_t* ids_out, int32_t* n_out,
                           volatile const int32_t* cancel);

/* ---- benchmark and profiling exports (no counterpart in the reference, which has no device) ---- */

/* Runs `steps` decode steps of the N sequences seqs[0..N) with token ids already on the device (the same ids every
 * step, taken from a seeded draw), no host copies, and returns the device time of the whole loop measured with CUDA
 * events on the model's stream. Sequence lengths advance by `steps`. */
int32_t wl_bench_decode(wl_model* model, wl_seq* const* seqs, int32_t N, int32_t steps, double* device_ms);
/* No counterpart in the reference: the Q4_K matvec launches of one decode step of T rows (1..8; the step's weights,
 * shapes, pairings and order), captured into a CUDA graph and replayed `steps` times alone, for the dominant kernel's
 * rate inside a step. Returns the device milliseconds of the replays (the maximum over the GPUs of a tensor-parallel
 * model) and the algorithmic bytes per step of those launches (this GPU's share). Outputs go to the model's scratch
 * rows; sequences are untouched. */
int32_t wl_bench_matvecs(wl_model* model, int32_t T, int32_t steps, double* device_ms, double* bytes_per_step);
/* on != 0 records CUDA events around every matvec/matmul launch (and clears the counters); 0 stops. */
int32_t wl_profile(wl_model* model, int32_t on);
/* The counters of weight format `type` (see wl_profile_entry). */
int32_t wl_profile_get(wl_model* model, int32_t type, wl_profile_entry* out);

/* ---- kernel-level exports for tests and benchmarks (device pointers, stream = cudaStream_t or NULL) ---- */

/* No counterpart in the reference. Failure detection of the tensor-parallel all-reduce without a GPU fault: runs the
 * all-reduce's consumer kernel on `device` against a peer rank that never pushes its partial (elements nothing
 * writes), its wait limited to wait_ms. The wait gives up, the kernel returns, and the call returns WL_ETIMEDOUT with the device still
 * usable, which is what a rank sees when a peer dies between steps. (Real waits are limited to 10 s.) */
int32_t wl_selftest_allreduce_timeout(int32_t device, int32_t wait_ms);

/* The greedy choice of wl_forward_argmax on `rows` rows of V device floats: dev_ids[r] = the lowest index of row r's
 * largest value (Argmax, src/Engine.cs:329-334; a NaN at index 0 gives 0). Synchronous on `stream`. */
int32_t wl_argmax(const float* dev_logits, int32_t V, int32_t rows, int32_t* dev_ids, void* stream);

/* Sampler.Sample of the sampled forward calls on V device floats: *dev_id = the chosen id. Synchronous on `stream`;
 * allocates its workspace (about 48 bytes a logit) for the call. */
int32_t wl_sample(const float* dev_logits, int32_t V, double temperature, double top_p, double draw, int32_t* dev_id,
                  void* stream);

/* Synchronises `device` and reports whether a device-side wait of a kernel-level export (wl_matvec, wl_matvec_tiles,
 * wl_matvec_static, wl_gemm_tiles, wl_matmul) gave up since the last report: WL_ETIMEDOUT (and the code) if one did,
 * else WL_OK. The waits are bounded at 2 s of device time, so this is a stalled copy, not a slow one. The model's own
 * calls report such a wait themselves. */
int32_t wl_kernel_status(int32_t device);

/* Transformer.Route (src/Transformer.cs:315-340) on the device for T tokens of n <= 256 router logits (device
 * floats, [T][n]): dev_sel[t*k + j] = the j-th expert picked, dev_wts[t*k + j] = its probability (renormalised over
 * the k picks when renorm != 0), k <= 32. Synchronous on `stream`. */
int32_t wl_route(const float* dev_logits, int32_t T, int32_t n, int32_t k, int32_t renorm, int32_t* dev_sel,
                 float* dev_wts, void* stream);

/* Quants.DecodeRow (src/Quants.cs:32-52, src/IQuants.cs:27-42): n values of `type` to fp32, bit-exact. */
int32_t wl_dequant(int32_t type, const void* dev_blocks, int64_t n, float* dev_out, void* stream);
/* Transformer.MatMulEach / Quants.DotRow (src/Transformer.cs:544-561, src/Quants.cs:67-187): y[t*rows + r] =
 * W[r] . x[t] for t < ncols (1..8), fused dequant-dot, fp32 accumulate. Every column is computed as if alone. */
int32_t wl_matvec(int32_t type, const void* dev_w, int32_t rows, int32_t cols, const float* dev_x, int32_t ncols,
                  float* dev_y, void* stream);
/* No counterpart in the reference. A Q4_K matvec (16-byte aligned weights and dev_x, cols a multiple of 256) with
 * wl_matvec's arguments, for callers that cannot let a call allocate device memory: its scratch (an error word and
 * the prepared activations of up to 8 columns) is a static device array of this library (WL_MATVEC_STATIC_MAX_COLS
 * columns, about 1 MB on every device that loads the library, held until exit), so the call makes no
 * cudaMalloc/cudaFree. It runs the tensor-core kernel on the GGUF rows through a TMA tensor map (wl_matvec repacks the
 * weights into tiles first); the results match wl_matvec's within the matvec tolerance (1e-4 relative L2). cols
 * above the limit or other formats return WL_EINVAL / WL_EUNSUPPORTED (use wl_matvec). The first call on each device
 * looks up the array's address with cudaGetSymbolAddress and sets the shared-memory attribute of all its kernel
 * instantiations: make it before any stream capture. The array starts at zero when the library loads; a kernel whose
 * bounded wait gives up sets its error word, which stays set until wl_kernel_status reads and clears it. Calls share
 * one scratch per device and leave their prepared activations in it, so calls that may overlap on the GPU
 * (different streams, or threads without ordering) race: order them on one stream. */
#define WL_MATVEC_STATIC_MAX_COLS 32768
int32_t wl_matvec_static(int32_t type, const void* dev_w, int32_t rows, int32_t cols, const float* dev_x,
                         int32_t ncols, float* dev_y, void* stream);
/* No counterpart in the reference: the tile-major weight layout the tensor-core matvec reads (Q4_K, Q6_K, Q8_0,
 * IQ4_XS and IQ2_XXS, cols a multiple of 256; every 16 rows x one 256-value superblock contiguous). The model repacks its weights this way once at load;
 * these let a caller do the same and then run matvecs without a per-call repack. wl_tiles_size gives the bytes
 * (rows rounded up to 16), wl_make_tiles fills dev_tiles (16-byte aligned) from GGUF rows, wl_matvec_tiles is
 * wl_matvec on the tiles (dev_x 16-byte aligned). Other formats return WL_EUNSUPPORTED. */
int32_t wl_tiles_size(int32_t type, int32_t rows, int32_t cols, int64_t* bytes);
int32_t wl_make_tiles(int32_t type, const void* dev_w, int32_t rows, int32_t cols, void* dev_tiles, void* stream);
int32_t wl_matvec_tiles(int32_t type, const void* dev_tiles, int32_t rows, int32_t cols, const float* dev_x,
                        int32_t ncols, float* dev_y, void* stream);
/* No counterpart in the reference: the standalone rate of the decode matvec. The activations (ncols of 1..8) are
 * prepared once, then `iters` wl_matvec_tiles launches over the tile buffers dev_tiles[i % copies] (each made by
 * wl_make_tiles from a rows x cols matrix; several copies whose total exceeds L2 keep the reads in HBM) run back to
 * back as one CUDA graph on an internal stream, as they follow each other inside a decode step; device_ms is the
 * CUDA-event time of the whole graph. dev_y receives the last launch's product. */
int32_t wl_bench_matvec_tiles(int32_t type, const void* const* dev_tiles, int32_t copies, int32_t rows, int32_t cols,
                              const float* dev_x, int32_t ncols, float* dev_y, int32_t iters, double* device_ms,
                              void* stream);
/* No counterpart in the reference: the tcgen05 GEMM (Q4_K only) on tile-major weights made by wl_make_tiles, for
 * T > 8 rows: dev_y[t*rows + r] = W[r] . dev_x[t]. The activations' bf16 hi/lo planes go to a scratch the library
 * keeps per device (grown on demand). Other formats return WL_EUNSUPPORTED. */
int32_t wl_gemm_tiles(int32_t type, const void* dev_tiles, int32_t rows, int32_t cols, const float* dev_x, int32_t T,
                      float* dev_y, void* stream);
/* Transformer.MatMul for T input rows (src/Transformer.cs:483-537): path 0 = the model's default (T > 8 rows of Q4_K
 * on the tcgen05 GEMM, else the integer tensor-core matvec in 8-column chunks where the format has one), 1 = fp32
 * CUDA cores, 2 = the integer tensor-core matvec in 8-column chunks. */
int32_t wl_matmul(int32_t type, const void* dev_w, int32_t rows, int32_t cols, const float* dev_x, int32_t T,
                  float* dev_y, int32_t path, void* stream);
/* Synthetic weight generator of wl_open_synthetic for one tensor (rows x cols of `type`: F32, F16, Q8_0, Q4_K or
 * Q6_K). F32 values are offset + sigma*z; other types quantize sigma*z. */
int32_t wl_synth_tensor(int32_t type, uint64_t seed, uint32_t tensor_id, int64_t rows, int64_t cols, float sigma,
                        float offset, void* dev_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif
