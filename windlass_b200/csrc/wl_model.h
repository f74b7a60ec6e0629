// The device-resident decoder: Transformer.cs's Forward / ForwardBatch / Truncate / NewSequence semantics on one
// GPU. Weights live in one device arena (resident) or stream through two device slots from pinned host memory;
// activations stay on the device for the whole pass; the host only uploads token ids and downloads logits.
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include "../../include/windlass.h"
#include "wl_kernels.h"
#include "wl_nccl.h"

namespace wl {

class Gguf;

// One weight tensor on the device. For stacked MoE tensors [cols, rows, experts] `rows` counts one expert's rows.
struct Weight {
    int type = -1;
    int rows = 0, cols = 0, experts = 1;
    int64_t row_bytes = 0, bytes = 0;
    uint8_t* d = nullptr;
    int row_base = 0;            // first row of this view inside the tiles (an expert slice)
    uint8_t* tiles = nullptr;    // Q4_K / Q6_K repacked into 16-row tiles for the tensor-core matvec (all experts)
    bool streamed_tiles = false; // streamed in tile layout only: d holds tiles, not GGUF rows
    bool present() const { return d != nullptr; }
    const uint8_t* expert(int e) const { return d + (int64_t)e * rows * row_bytes; }
};

// A vector (norm weight, bias) decoded to fp32 on the device (Transformer.Vector, src/Transformer.cs:435-440).
struct Vec {
    float* d = nullptr;
    int n = 0;
    bool present() const { return d != nullptr; }
};

struct LayerW {
    Vec attn_norm, qb, kb, vb, q_norm, k_norm, post_attn_norm, ffn_norm, post_ffw_norm;
    Weight q, k, v, o, gate, up, down, router, gate_exps, up_exps, down_exps, sh_gate, sh_up, sh_down, sh_gate_inp;
    bool moe = false;
};

// ModelConfig (src/ModelConfig.cs:12-36): the fields the forward pass reads.
struct Config {
    std::string arch;
    int layers = 0, embd = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0, context_length = 0, rope_dims = 0;
    float rms_eps = 1e-5f, rope_base = 10000.f, rope_freq_scale = 1.f;
    bool rope_neox = false, qk_norm = false, qk_norm_full = false, post_norms = false, tied = false;
    float embedding_scale = 0, residual_scale = 0, attention_scale = 0, logit_scale = 0;
    int expert_count = 0, expert_used = 0, expert_ff = 0, shared_expert_ff = 0;
    bool expert_weights_norm = false;
    int qdim() const { return heads * head_dim; }
    int kvdim() const { return kv_heads * head_dim; }
};

class Model;

// Sequence (src/Batch.cs:13-36): one request's fp16 KV cache in device memory, [2][layers][capacity][kv_dim].
struct Seq {
    Model* model = nullptr;
    uint16_t* kv = nullptr;
    int capacity = 0;
    int length = 0;
};

struct Stats {
    int64_t bytes_h2d = 0, expert_runs = 0, forward_calls = 0, batch_calls = 0, tokens = 0;
    double last_forward_ms = 0;
};

class Model {
public:
    static Model* open_file(const std::string& path, const wl_options& opt);
    static Model* open_synthetic(const wl_synth_spec& spec, const wl_options& opt);
    ~Model();

    Seq* new_seq();
    void free_seq(Seq* s);
    Seq* own() { return own_; }

    // Transformer.Forward / ForwardBatch. out is host memory. Return WL_OK or WL_CANCELLED; throw wl::Error.
    int32_t forward(Seq* seq, const int32_t* tokens, int T, int pos0, bool all_logits, float* out,
                    volatile const int32_t* cancel, wl_progress_fn progress, void* user);
    int32_t forward_batch(Seq* const* seqs, const int32_t* tokens, int N, float* out, volatile const int32_t* cancel,
                          wl_progress_fn progress, void* user);
    // The same passes with the greedy choice made on the device: ids (host) gets each returned row's argmax
    // (Sampler.Sample at temperature 0, src/Engine.cs:356-360) instead of its logits.
    int32_t forward_argmax(Seq* seq, const int32_t* tokens, int T, int pos0, bool all_rows, int32_t* ids,
                           volatile const int32_t* cancel, wl_progress_fn progress, void* user);
    int32_t forward_batch_argmax(Seq* const* seqs, const int32_t* tokens, int N, int32_t* ids,
                                 volatile const int32_t* cancel, wl_progress_fn progress, void* user);
    // The same passes with Sampler.Sample (src/Engine.cs:361-380) made on the device: returned row r is sampled with
    // temperature[r], top_p[r] and the host's uniform draw[r] in [0, 1) (its rng.NextDouble(), unused at temperature
    // <= 0), and ids gets the chosen id.
    struct SampleRows {
        const double* temperature;
        const double* top_p;
        const double* draw;
    };
    int32_t forward_sample(Seq* seq, const int32_t* tokens, int T, int pos0, const SampleRows& sr, int32_t* id,
                           volatile const int32_t* cancel, wl_progress_fn progress, void* user);
    int32_t forward_batch_sample(Seq* const* seqs, const int32_t* tokens, int N, const SampleRows& sr, int32_t* ids,
                                 volatile const int32_t* cancel, wl_progress_fn progress, void* user);
    // One pass over several sequences' new tokens at once (a decode step that prompts join: continuous batching):
    // sequence i takes counts[i] tokens at its next positions, tokens holding them sequence after sequence; out (or
    // ids) gets each sequence's last row, in sequence order. Each row attends to its own sequence only.
    int32_t forward_mixed(Seq* const* seqs, const int32_t* counts, int N, const int32_t* tokens, float* out,
                          int32_t* ids, volatile const int32_t* cancel, wl_progress_fn progress, void* user);
    // Greedy decode chained on the device (the loop of LayeredBackend.Generate, src/Engine.cs:187-203, at
    // temperature 0 without guesses): step s forwards `token` (s = 0) or ids[s-1] at the sequence's next position and
    // writes the argmax to ids[s]; the argmax becomes the next step's token in device memory, so up to `chunk` steps
    // run back to back before the host reads their ids. Stops after a stop id or max_new steps; *n = steps kept, and
    // the sequence grows by *n.
    int32_t generate_greedy(Seq* seq, int32_t token, int max_new, const int32_t* stop, int n_stop, int chunk,
                            int32_t* ids, int32_t* n, volatile const int32_t* cancel);

    // The model's shape; under tensor parallelism heads and kv_heads are this rank's share (full_config() has the
    // whole model's).
    const Config& config() const { return c_; }
    const Config& full_config() const { return full_; }
    int tp_size() const { return tp_size_; }
    int tp_rank() const { return tp_rank_; }
    bool tp_fused() const { return ar_on_; }
    // This shard leaves its group without the collectives of an orderly close (its peers are gone or leave the same
    // way, and no step has run): used when a group fails to open.
    void detach_group() { opened_ = false; }
    int max_context() const { return max_context_; }
    const Stats& stats() const { return stats_; }
    int64_t graph_launches() const { return graph_launches_; }
    int64_t weight_bytes() const { return weight_bytes_; }
    int64_t device_bytes() const;
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    // y[T][rows] = W x[T][cols] on the model's stream (row t at y + t*ldy, ldy 0 = rows); path 0 chooses by T (the
    // forward pass's own rule).
    void matmul(const Weight& w, const float* x, int T, float* y, int path = 0, bool reuse_x = false, int64_t ldy = 0);
    // ya = A x and yb = B x for two matrices with the same input (q and k, gate and up): one tensor-core launch for
    // decode steps when both are tiled Q4_K, else two matmuls. Each row's result is what matmul gives.
    void matmul2(const Weight& a, const Weight& b, const float* x, int T, float* ya, float* yb);

    // Device-resident decode loop for benchmarks: returns the device milliseconds of `steps` steps.
    double bench_decode(Seq* const* seqs, int N, int steps);
    double bench_matvecs(int T, int steps, double* bytes);
    void set_profiling(bool on);
    wl_profile_entry profile(int type);

private:
    struct ProfileMark {
        cudaEvent_t start, stop;
        int type;
        double bytes;
    };
    struct GraphEntry {
        int T, first, gen;
        cudaGraphExec_t exec;
        int64_t nodes;
    };
    bool graphable(int T) const;
    bool graph_ready(int T, int first);
    bool graph_step(int T, int first);
    void drop_graphs();
    void flush_profile();
    void build_maps();
    void check_device_error();
    int profile_begin();
    void profile_end(int mark, int kind, double bytes);
    void upload_step(int T, const RowKV* rows, const int32_t* pos, const int32_t* tokens);
    void step_device(int T, int first, int max_n);
    Model() = default;
    void init_device(const wl_options& opt);
    void init_tp(const wl_options& opt);
    void all_reduce(float* buf, int64_t n);
    void init_fused_ar(const wl_options& opt);
    void close_fused_ar();
    void matmul_reduce(const Weight& w, const float* x, int T);
    bool pending_ar_in(int T, int row0, k::ArIn* in);
    k::ArOut ar_out(int idx) const;
    void begin_step(int T);
    bool stop_requested(volatile const int32_t* cancel);
    void finish_open();
    // layer streaming (wl_stream.cpp)
    int stage_of_name(const std::string& name) const;
    void plan_streaming(const std::vector<int64_t>& raw_upper, const std::vector<int64_t>& slot_upper);
    uint8_t* weight_alloc(int64_t bytes);
    void end_stage(int l, const std::vector<Weight*>& ws);
    void finish_streaming();
    void issue_copy(int l);
    void stage_acquire(int l);
    void stage_release(int l);
    void free_streaming();
    void load_from_gguf(const Gguf& g);
    void build_rope_table(const float* rope_freqs, int n_rope_freqs);
    void reserve(Seq* s, int positions);
    void ensure_workspace(int T, int logit_rows);
    void layer(int l, int T, int max_n);
    void pre_norm(int T, const Vec& w, bool prep_for_mma);
    void ffn_dense(const LayerW& L, int T);
    void ffn_moe(const LayerW& L, int T);
    bool moe_on_device(const LayerW& L, int T) const;
    void ffn_moe_device(const LayerW& L, int T);
    void head(int T, int first);
    // One pass; the rows from first_logit_row on come back as logits (out) or as their argmax (ids).
    int32_t run(int T, const std::vector<RowKV>& rows, const std::vector<int32_t>& pos, const int32_t* tokens,
                int first_logit_row, float* out, int32_t* ids, volatile const int32_t* cancel, wl_progress_fn progress,
                void* user);
    int32_t forward_impl(Seq* seq, const int32_t* tokens, int T, int pos0, bool all_logits, float* out, int32_t* ids,
                         volatile const int32_t* cancel, wl_progress_fn progress, void* user);
    int32_t forward_batch_impl(Seq* const* seqs, const int32_t* tokens, int N, float* out, int32_t* ids,
                               volatile const int32_t* cancel, wl_progress_fn progress, void* user);
    uint8_t* arena_alloc(int64_t bytes);

    Config c_, full_;
    int device_ = 0;
    // tensor parallelism: this rank's share of rows (q/k/v, gate/up, the head) and columns (o, down)
    int tp_size_ = 1, tp_rank_ = 0;
    // the routed experts this GPU holds: e_lo_ .. e_lo_ + e_n_ - 1 (all of them on one GPU)
    int e_lo_ = 0, e_n_ = 1 << 30;
    std::unique_ptr<Comm> comm_;
    int vocab_part_ = 0;                  // output-head rows per rank (the last rank's may hold fewer real rows)
    float* logits_part_ = nullptr;        // [rows][vocab_part_] this rank's head rows
    float* logits_all_ = nullptr;         // [tp][rows][vocab_part_] every rank's, after the all-gather
    int32_t* flag_d_ = nullptr;           // the cancel flag agreed over ranks (device, pinned host)
    int32_t* flag_h_ = nullptr;
    // the fused all-reduce (k::ArOut / k::ArIn): this rank's buffer and every peer's, mapped through CUDA IPC
    uint8_t* ar_buf_ = nullptr;
    uint8_t* ar_peer_[k::AR_MAX_RANKS] = {};
    bool ar_ipc_[k::AR_MAX_RANKS] = {};   // mapped through CUDA IPC (another process), else a pointer in this one
    bool ar_on_ = false;
    int ar_idx_ = 0;                      // fused all-reduces enqueued so far in the current step
    int pending_ar_ = -1;                 // index of the all-reduce whose sum the next norm consumes, or -1
    const k::ArOut* ar_out_ = nullptr;    // set while matmul_reduce runs: the Q4_K decode matvec pushes into it
    bool ar_out_done_ = false;            // the matvec pushed (else matmul_reduce pushes the staged partial)
    int max_context_ = 0;
    int max_batch_ = 64;
    int prefill_path_ = 0;
    bool each_token_ = false;             // a ForwardBatch step: every row computed as if alone (no GEMM)
    cudaStream_t stream_ = nullptr;
    // decode steps run the v matvec on side_ (forked after the pre-norm, joined before RoPE) beside q and k
    cudaStream_t side_ = nullptr;
    cudaEvent_t fork_ev_ = nullptr, join_ev_ = nullptr;
    std::vector<LayerW> L_;
    Weight embd_, output_;
    Vec out_norm_;
    float* rope_table_ = nullptr;         // [max_context][rope_dims] cos/sin pairs
    Seq* own_ = nullptr;
    Stats stats_;
    int64_t weight_bytes_ = 0;

    // layer streaming (wl_options.resident = 0): per stage (each layer, then the head) its weights in pinned host
    // memory, laid out as the kernels read them; two device slots, stage l in slot l % 2
    struct StageWeight {
        Weight* w;
        int64_t off;
        bool tiled;
    };
    // file-backed streaming: a stage's tensor as the reader fetches it (its GGUF bytes at file_off; tiled ones land
    // in the staging area at raw_off and are repacked into the slot, the rest go to the slot directly)
    struct FileItem {
        int64_t file_off, bytes, raw_off, slot_off;
        Weight* w;
        bool tiled;
        int rows_total;
    };
    struct Stage {
        std::vector<StageWeight> ws;
        std::vector<FileItem> file;
        uint8_t* host = nullptr;
        int64_t bytes = 0;
    };
    bool streamed_ = false;
    bool stream_file_ = false;            // stages read from the GGUF file at every use (wl_options.stream_file)
    std::string file_path_;
    // the tensors uploaded into the staging area while the current stage loads: staging offset -> (file offset, bytes)
    std::vector<std::pair<int64_t, std::pair<int64_t, int64_t>>> file_src_;
    struct FileReader;
    FileReader* reader_ = nullptr;
    void reader_loop();
    void reader_fetch(int l);
    void reader_wait(int l);
    bool opened_ = false;                 // open completed: closing meets the other ranks in collectives
    std::vector<Stage> stages_;
    int cur_stage_ = -1;                  // the stage being loaded (-1: resident weights)
    uint8_t* staging_ = nullptr;
    int64_t staging_size_ = 0, staging_used_ = 0;
    uint8_t* slot_[2] = {nullptr, nullptr};
    int64_t slot_bytes_ = 0;
    int slot_stage_[2] = {-1, -1};        // the stage each slot holds (or is being copied)
    cudaStream_t copy_stream_ = nullptr;
    cudaEvent_t copied_[2] = {nullptr, nullptr}, freed_[2] = {nullptr, nullptr};

    // device arena holding every weight
    uint8_t* arena_ = nullptr;
    int64_t arena_size_ = 0, arena_used_ = 0;
    std::vector<void*> extra_allocs_;

    // workspaces (grown on demand)
    int ws_T_ = 0, ws_logit_rows_ = 0;
    float *x_ = nullptr, *xn_ = nullptr, *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *att_ = nullptr, *o_ = nullptr;
    float *g_ = nullptr, *u_ = nullptr, *logits_ = nullptr, *router_ = nullptr, *wts_ = nullptr;
    float *xe_ = nullptr, *ye_ = nullptr, *ge_ = nullptr, *ue_ = nullptr, *moe_out_ = nullptr, *sh_gl_ = nullptr;
    int32_t *tok_d_ = nullptr, *pos_d_ = nullptr, *sel_ = nullptr, *bad_d_ = nullptr, *etok_d_ = nullptr;
    // greedy selection: per logit row its argmax, merge key and block counter (zero between launches), and the
    // chained decode's ids with their pinned host copy
    int32_t* ids_d_ = nullptr;
    unsigned long long* amax_key_ = nullptr;
    unsigned* amax_count_ = nullptr;
    int32_t* h_ids_ = nullptr;
    // device sampling: the rows' options during a forward_sample / forward_batch_sample call, and the sampler's
    // workspace (one row's, made at the first sampled call; its first 256 bytes stay zero between rows)
    const SampleRows* sampling_ = nullptr;
    void* sample_ws_ = nullptr;
    int32_t* gen_d_ = nullptr;
    int32_t* h_gen_ = nullptr;
    float* ew_d_ = nullptr;
    RowKV* rows_d_ = nullptr;
    // pinned host staging
    int32_t* h_tok_ = nullptr;
    int32_t* h_pos_ = nullptr;
    RowKV* h_rows_ = nullptr;
    int32_t* h_sel_ = nullptr;
    float* h_wts_ = nullptr;
    int32_t* h_etok_ = nullptr;
    float* h_ew_ = nullptr;
    int h_cap_ = 0;
    // activations prepared for the tensor-core matvec (k::xprep), and what they were prepared from
    // the device-side mixture-of-experts path of decode steps: per (token, chosen expert) pair its gate, up and
    // down outputs, the prepared SwiGLU outputs, and a device count of the experts run
    float *pg_ = nullptr, *pu_ = nullptr, *py_ = nullptr;
    void* pprep_ = nullptr;
    int pair_cap_ = 0;
    unsigned long long* expert_count_d_ = nullptr;
    void* gemm_buf_ = nullptr;          // the tcgen05 GEMM's activation planes
    size_t gemm_buf_bytes_ = 0;
    void* xprep_buf_ = nullptr;
    float* att_part_ = nullptr;         // split-range attention partials
    int* err_d_ = nullptr;              // device error word of the bounded waits
    const float* prep_x_ = nullptr;
    int prep_cols_ = 0, prep_nc_ = 0;
    bool pending_residual_ = false;     // x += o_ not yet applied (done by the next norm)
    bool pending_moe_ = false;          // ... and o_ is the expert combine of moe_in_, computed by that norm
    k::MoeIn moe_in_{};
    // CUDA graphs of decode steps
    bool use_graphs_ = true;
    std::vector<GraphEntry> graphs_;
    int ws_gen_ = 0;                    // bumped whenever a workspace the graphs point into is reallocated
    int64_t graph_launches_ = 0;        // kernels launched by graph replays
    // profiling
    bool profiling_ = false;
    std::vector<ProfileMark> marks_;
    std::vector<cudaEvent_t> event_pool_;
    wl_profile_entry prof_[64] = {};
};

}  // namespace wl
