// Device-resident decoder forward: Transformer.cs (Forward, ForwardBatch, Layer, Head, MoeFfn), ModelConfig.From and
// the stage name binding of LayerStream.Bind, re-designed for one GPU: weights in one HBM arena, activations and the
// fp16 KV caches on the device, one CUDA stream per model, the host touching only token ids and logits.
#include "wl_model.h"
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <unistd.h>
#include "wl_common.h"
#include "wl_gguf.h"

namespace wl {

namespace {
template <typename T> T* dalloc(int64_t n)
{
    void* p = nullptr;
    if (n <= 0) n = 1;
    WL_CUDA(cudaMalloc(&p, sizeof(T) * (size_t)n));
    return (T*)p;
}
template <typename T> void dfree(T*& p)
{
    if (p) cudaFree((void*)p);
    p = nullptr;
}
template <typename T> T* halloc(int64_t n)
{
    void* p = nullptr;
    if (n <= 0) n = 1;
    WL_CUDA(cudaMallocHost(&p, sizeof(T) * (size_t)n));
    return (T*)p;
}
template <typename T> void hfree(T*& p)
{
    if (p) cudaFreeHost((void*)p);
    p = nullptr;
}
}  // namespace

// ---------------------------------------------------------------------------------------------------------------------
// open / close
// ---------------------------------------------------------------------------------------------------------------------
static int tp_size_of(const wl_options& opt);

void Model::init_device(const wl_options& opt)
{
    streamed_ = opt.resident == 0;
    stream_file_ = streamed_ && opt.stream_file == 1;
    if (opt.stream_file != 0 && opt.stream_file != 1) WL_THROW(WL_EINVAL, "stream_file must be 0 or 1.");
    if (opt.stream_file == 1 && !streamed_) WL_THROW(WL_EINVAL, "stream_file needs resident = 0 (streamed layers).");
    if (stream_file_ && tp_size_of(opt) > 1)
        WL_THROW(WL_EUNSUPPORTED, "stream_file streams one GPU's layers; tensor parallelism keeps its shards resident or in pinned memory.");
    if (streamed_ && opt.prefill_path == 1)
        WL_THROW(WL_EUNSUPPORTED, "Streamed layers carry the tensor-core layout only; prefill_path 1 (CUDA cores) needs resident weights.");
    device_ = opt.device;
    WL_CUDA(cudaSetDevice(device_));
    k::init_tables();
    WL_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    WL_CUDA(cudaStreamCreateWithFlags(&side_, cudaStreamNonBlocking));
    WL_CUDA(cudaEventCreateWithFlags(&fork_ev_, cudaEventDisableTiming));
    WL_CUDA(cudaEventCreateWithFlags(&join_ev_, cudaEventDisableTiming));
    max_batch_ = opt.max_batch > 0 ? opt.max_batch : 64;
    use_graphs_ = opt.use_graphs != 0;
    prefill_path_ = opt.prefill_path;
}

// Tensor parallelism (tp_size > 1): checks the shape can be split, makes c_ this rank's share of the heads and joins
// the NCCL group (blocking until every rank has joined). Called once the configuration is known, before any weight
// is loaded, so a model every rank would refuse fails on every rank before the group forms.
static int tp_size_of(const wl_options& opt)
{
    return opt.size >= (int32_t)sizeof(wl_options) && opt.tp_size > 1 ? opt.tp_size : 1;
}

// The checks of a tensor-parallel split that need no device: they run before the device is touched, so a model that
// every rank would refuse fails the same way on every rank, before any rank waits for the group to form.
static void check_tp(const Config& c, const wl_options& opt)
{
    const int G = tp_size_of(opt);
    if (G == 1) return;
    const std::string g = std::to_string(G);
    if (opt.tp_rank < 0 || opt.tp_rank >= G) WL_THROW(WL_EINVAL, "tp_rank must be 0.." + std::to_string(G - 1) + ".");
    if (c.expert_count % G)
        WL_THROW(WL_EUNSUPPORTED, "Tensor parallelism over " + g + " GPUs places whole experts on each GPU and needs an "
                                  "expert count divisible by " + g + " (" + std::to_string(c.expert_count) + " experts).");
    if (c.qk_norm_full || c.post_norms)
        WL_THROW(WL_EUNSUPPORTED, "Tensor parallelism does not split " + c.arch + " (its QK-norm spans every head).");
    if (c.heads % G || c.kv_heads % G)
        WL_THROW(WL_EUNSUPPORTED, "Tensor parallelism over " + g + " GPUs needs head counts divisible by " + g + " (" +
                                  std::to_string(c.heads) + " heads, " + std::to_string(c.kv_heads) + " KV heads).");
    if (!k::attention_supported(c.heads / G, c.kv_heads / G, c.head_dim))
        WL_THROW(WL_EUNSUPPORTED, "Tensor parallelism over " + g + " GPUs leaves an unsupported attention shape per GPU.");
    const int vp = (c.vocab + G - 1) / G;
    if ((int64_t)vp * (G - 1) >= c.vocab) WL_THROW(WL_EUNSUPPORTED, "The vocabulary is too small to split over " + g + " GPUs.");
}

// Tensor parallelism (tp_size > 1): makes c_ this rank's share of the heads and joins the NCCL group (blocking until
// every rank has joined). Called once the configuration is known and checked, before any weight is loaded.
void Model::init_tp(const wl_options& opt)
{
    full_ = c_;
    check_tp(c_, opt);
    tp_size_ = tp_size_of(opt);
    tp_rank_ = tp_size_ > 1 ? opt.tp_rank : 0;
    if (tp_size_ == 1) return;
    c_.heads /= tp_size_;
    c_.kv_heads /= tp_size_;
    if (c_.expert_count > 0) {
        e_n_ = c_.expert_count / tp_size_;
        e_lo_ = tp_rank_ * e_n_;
    }
    vocab_part_ = (c_.vocab + tp_size_ - 1) / tp_size_;
    flag_d_ = dalloc<int32_t>(1);
    flag_h_ = halloc<int32_t>(1);
    comm_.reset(new Comm(opt.tp_id, tp_size_, tp_rank_));
    init_fused_ar(opt);
}

// Maps every rank's all-reduce buffer into this process. Ranks exchange (process id, device, pointer, CUDA IPC
// handle) with an NCCL all-gather: a peer in another process is mapped through its IPC handle, a peer in this process
// (one wl_model spanning several GPUs) is reached through its pointer once peer access to its device is on. All ranks
// agree on the outcome: if any rank cannot reach a peer, every rank keeps NCCL for all its all-reduces.
void Model::init_fused_ar(const wl_options& opt)
{
    const int G = tp_size_;
    if (opt.tp_nccl_only || G > k::AR_MAX_RANKS || 2 * c_.layers + 2 > k::AR_STEP || !k::norm_prep_supported(c_.embd)) return;
    const size_t bytes = k::ar_buffer_bytes(c_.embd);
    ar_buf_ = dalloc<uint8_t>((int64_t)bytes);
    WL_CUDA(cudaMemset(ar_buf_, 0, bytes));
    struct PeerRec {
        cudaIpcMemHandle_t handle;
        uint64_t ptr;
        int64_t pid;
        int32_t device, ok;
        uint8_t pad[128 - 64 - 24];
    };
    static_assert(sizeof(PeerRec) == 128, "peer record size");
    PeerRec mine{};
    mine.ok = cudaIpcGetMemHandle(&mine.handle, ar_buf_) == cudaSuccess;
    cudaGetLastError();
    mine.ptr = (uint64_t)(uintptr_t)ar_buf_;
    mine.pid = (int64_t)getpid();
    mine.device = device_;
    uint8_t* hd = dalloc<uint8_t>(128 * G);
    std::vector<PeerRec> all(G);
    WL_CUDA(cudaMemcpy(hd + 128 * tp_rank_, &mine, 128, cudaMemcpyHostToDevice));
    comm_->allgather(hd + 128 * tp_rank_, hd, 128, stream_);
    WL_CUDA(cudaStreamSynchronize(stream_));
    WL_CUDA(cudaMemcpy(all.data(), hd, 128 * (size_t)G, cudaMemcpyDeviceToHost));
    dfree(hd);
    int failed = 0;
    for (int g = 0; g < G && !failed; ++g) {
        ar_ipc_[g] = false;
        if (g == tp_rank_) { ar_peer_[g] = ar_buf_; continue; }
        if (all[g].pid == mine.pid) {
            int can = 0;
            if (cudaDeviceCanAccessPeer(&can, device_, all[g].device) != cudaSuccess || !can) { failed = 1; break; }
            const cudaError_t e = cudaDeviceEnablePeerAccess(all[g].device, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) failed = 1;
            cudaGetLastError();
            if (!failed) ar_peer_[g] = (uint8_t*)(uintptr_t)all[g].ptr;
            continue;
        }
        void* p = nullptr;
        if (!all[g].ok || cudaIpcOpenMemHandle(&p, all[g].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            failed = 1;
        } else {
            ar_peer_[g] = (uint8_t*)p;
            ar_ipc_[g] = true;
        }
    }
    *flag_h_ = failed;
    WL_CUDA(cudaMemcpy(flag_d_, flag_h_, sizeof(int32_t), cudaMemcpyHostToDevice));
    comm_->allreduce_max(flag_d_, 1, stream_);
    WL_CUDA(cudaStreamSynchronize(stream_));
    WL_CUDA(cudaMemcpy(flag_h_, flag_d_, sizeof(int32_t), cudaMemcpyDeviceToHost));
    ar_on_ = *flag_h_ == 0;
    if (!ar_on_) {
        // every rank takes this path together, so the orderly close's collectives meet
        opened_ = true;
        close_fused_ar();
        opened_ = false;
    }
}

// Every rank stops using the buffers before any rank unmaps or frees its own (two NCCL barriers around the unmap).
void Model::close_fused_ar()
{
    if (!ar_buf_) return;
    // a model whose open did not complete has run no step: nothing reads the buffers, and its peers may be gone
    auto barrier = [&] {
        WL_CUDA(cudaStreamSynchronize(stream_));
        if (!opened_) return;
        comm_->allreduce_max(flag_d_, 1, stream_);
        WL_CUDA(cudaStreamSynchronize(stream_));
    };
    barrier();
    for (int g = 0; g < tp_size_; ++g) {
        if (g != tp_rank_ && ar_peer_[g] && ar_ipc_[g]) cudaIpcCloseMemHandle(ar_peer_[g]);
        ar_peer_[g] = nullptr;
        ar_ipc_[g] = false;
    }
    barrier();
    dfree(ar_buf_);
    ar_on_ = false;
}

// The output projection of a sublayer (o or down) summed over the tensor-parallel ranks into the next norm's input:
// for decode steps this rank's partial is pushed into every rank's all-reduce buffer (by the Q4_K decode matvec's
// epilogue, else staged and pushed by k::ar_push) and the next norm sums every rank's (k::ArIn), else the matvec
// writes o_ and NCCL all-reduces it. One GPU: the matvec into o_.
void Model::matmul_reduce(const Weight& w, const float* x, int T)
{
    const int E = c_.embd;
    if (ar_on_ && T <= k::AR_COLS && w.rows == E && ar_idx_ < k::AR_STEP) {
        const int idx = ar_idx_++;
        const k::ArOut ao = ar_out(idx);
        float* stage = reinterpret_cast<float*>(ar_buf_ + k::ar_slot_offset(idx, E));
        ar_out_ = &ao;
        ar_out_done_ = false;
        try {
            matmul(w, x, T, stage, 0, true, E);
        } catch (...) {
            ar_out_ = nullptr;
            throw;
        }
        ar_out_ = nullptr;
        if (!ar_out_done_) k::ar_push(stage, T, ao, stream_);
        pending_ar_ = idx;
        return;
    }
    matmul(w, x, T, o_, 0, true);
    all_reduce(o_, (int64_t)T * E);
}

// The producer side of fused all-reduce idx: every rank's pushed-element region.
k::ArOut Model::ar_out(int idx) const
{
    k::ArOut ao{};
    for (int g = 0; g < tp_size_; ++g)
        ao.ll[g] = reinterpret_cast<unsigned long long*>(ar_peer_[g] + k::ar_ll_offset(c_.embd));
    ao.epoch = reinterpret_cast<const unsigned long long*>(ar_buf_ + k::AR_EPOCH);
    ao.idx = idx;
    ao.G = tp_size_;
    ao.rank = tp_rank_;
    ao.E = c_.embd;
    return ao;
}

// The consumer side of the pending fused all-reduce for rows row0 .. row0+T-1; false when none is pending.
bool Model::pending_ar_in(int T, int row0, k::ArIn* in)
{
    if (pending_ar_ < 0) return false;
    (void)T;
    in->ll = reinterpret_cast<const unsigned long long*>(ar_buf_ + k::ar_ll_offset(c_.embd));
    in->epoch = reinterpret_cast<const unsigned long long*>(ar_buf_ + k::AR_EPOCH);
    in->err = err_d_;
    in->idx = pending_ar_;
    in->G = tp_size_;
    in->rank = tp_rank_;
    in->E = c_.embd;
    in->row0 = row0;
    in->wait_ns = k::AR_WAIT_NS;
    pending_ar_ = -1;
    return true;
}

// The start of every step: the embedding of its tokens (advancing the fused all-reduce epoch).
void Model::begin_step(int T)
{
    ar_idx_ = 0;
    pending_ar_ = -1;
    k::embed(embd_.type, embd_.d, embd_.row_bytes, embd_.rows, c_.embd, tok_d_, T, c_.embedding_scale, x_,
             bad_d_, stream_, ar_on_ ? reinterpret_cast<unsigned long long*>(ar_buf_ + k::AR_EPOCH) : nullptr);
    pending_residual_ = false;
    pending_moe_ = false;
}

// The cancel flag, polled between stages (Transformer.cs:99,158). Under tensor parallelism the ranks take the maximum
// of their flags, so all of them stop at the same stage and none waits in a collective the others skipped.
bool Model::stop_requested(volatile const int32_t* cancel)
{
    if (!cancel) return false;
    if (!comm_) return *cancel != 0;
    *flag_h_ = *cancel ? 1 : 0;
    WL_CUDA(cudaMemcpyAsync(flag_d_, flag_h_, sizeof(int32_t), cudaMemcpyHostToDevice, stream_));
    comm_->allreduce_max(flag_d_, 1, stream_);
    WL_CUDA(cudaMemcpyAsync(flag_h_, flag_d_, sizeof(int32_t), cudaMemcpyDeviceToHost, stream_));
    WL_CUDA(cudaStreamSynchronize(stream_));
    return *flag_h_ != 0;
}

// Sums a sublayer's partial outputs over the tensor-parallel ranks (no-op on one GPU).
void Model::all_reduce(float* buf, int64_t n)
{
    if (!comm_) return;
    const int mark = profile_begin();
    comm_->allreduce_sum(buf, n, stream_);
    profile_end(mark, WL_PROFILE_ALLREDUCE, 8.0 * n * (tp_size_ - 1) / tp_size_);
}

uint8_t* Model::arena_alloc(int64_t bytes)
{
    const int64_t a = (bytes + 255) / 256 * 256;
    if (arena_used_ + a > arena_size_) WL_THROW(WL_ENOMEM, "weight arena overflow");
    uint8_t* p = arena_ + arena_used_;
    arena_used_ += a;
    return p;
}

static std::string layer_name(int l, const char* s) { return "blk." + std::to_string(l) + "." + s; }

// ModelConfig.From (src/ModelConfig.cs:38-110).
static Config read_config(const Gguf& g)
{
    Config c;
    c.arch = g.get_string("general.architecture", "");
    static const char* archs[] = {"llama", "qwen2", "qwen3", "mixtral", "qwen2moe", "qwen3moe", "granite", "olmo2"};
    bool ok = false;
    for (const char* a : archs) ok |= c.arch == a;
    if (!ok)
        WL_THROW(WL_EUNSUPPORTED, "Model architecture '" + c.arch + "' is not supported. Windlass runs llama, qwen2, qwen3, "
                                  "mixtral, qwen2moe, qwen3moe, granite, olmo2.");
    const std::string a = c.arch + ".";
    c.layers = (int)g.get_int(a + "block_count", 0);
    c.embd = (int)g.get_int(a + "embedding_length", 0);
    c.heads = (int)g.get_int(a + "attention.head_count", 0);
    c.kv_heads = (int)g.get_int(a + "attention.head_count_kv", c.heads);
    c.head_dim = (int)g.get_int(a + "attention.key_length", c.heads ? c.embd / c.heads : 0);
    c.rope_dims = (int)g.get_int(a + "rope.dimension_count", c.head_dim);
    c.context_length = (int)g.get_int(a + "context_length", 4096);
    c.rms_eps = g.get_float(a + "attention.layer_norm_rms_epsilon", 1e-5f);
    c.rope_base = g.get_float(a + "rope.freq_base", 10000.f);
    c.rope_neox = c.arch == "qwen2" || c.arch == "qwen3" || c.arch == "qwen2moe" || c.arch == "qwen3moe" || c.arch == "olmo2";
    if (c.arch == "granite") {
        c.embedding_scale = g.get_float(a + "embedding_scale", 0.f);
        c.residual_scale = g.get_float(a + "residual_scale", 0.f);
        c.attention_scale = g.get_float(a + "attention.scale", 0.f);
        c.logit_scale = g.get_float(a + "logit_scale", 0.f);
    }
    c.post_norms = c.arch == "olmo2";
    c.qk_norm_full = c.arch == "olmo2";
    c.qk_norm = g.find("blk.0.attn_q_norm.weight") != nullptr;
    c.tied = g.find("output.weight") == nullptr;
    const std::string scaling = g.get_string(a + "rope.scaling.type", "none");
    const float factor = g.get_float(a + "rope.scaling.factor", 0.f);
    if (scaling == "linear" && factor > 0) c.rope_freq_scale = 1.f / factor;
    c.expert_count = (int)g.get_int(a + "expert_count", 0);
    if (c.expert_count > 0 && c.arch != "llama" && c.arch != "mixtral" && c.arch != "qwen2moe" && c.arch != "qwen3moe")
        WL_THROW(WL_EUNSUPPORTED, "Mixture-of-experts layers are supported for llama/mixtral, qwen2moe and qwen3moe, not '" + c.arch + "'.");
    if (c.expert_count == 0 && (c.arch == "qwen2moe" || c.arch == "qwen3moe"))
        WL_THROW(WL_EUNSUPPORTED, c.arch + " needs " + a + "expert_count.");
    if (c.expert_count > 0) {
        c.expert_used = (int)g.get_int(a + "expert_used_count", 0);
        if (c.expert_used < 1 || c.expert_used > c.expert_count)
            WL_THROW(WL_EUNSUPPORTED, a + "expert_used_count " + std::to_string(c.expert_used) + " must be 1.." + std::to_string(c.expert_count) + ".");
        bool norm = c.arch != "qwen2moe";
        if (g.has(a + "expert_weights_norm")) norm = g.get_bool(a + "expert_weights_norm", norm);
        c.expert_weights_norm = norm;
        if (c.expert_count > 256) WL_THROW(WL_EUNSUPPORTED, "more than 256 experts");
    }
    if (c.layers <= 0 || c.embd <= 0 || c.heads <= 0 || c.kv_heads <= 0) WL_THROW(WL_EUNSUPPORTED, "The model shape is incomplete.");
    if (c.heads % c.kv_heads != 0) WL_THROW(WL_EUNSUPPORTED, "head_count must be a multiple of head_count_kv.");
    if (c.rope_dims > c.head_dim || c.rope_dims % 2 != 0) WL_THROW(WL_EUNSUPPORTED, "Unsupported rope.dimension_count " + std::to_string(c.rope_dims) + ".");
    if (!k::attention_supported(c.heads, c.kv_heads, c.head_dim))
        WL_THROW(WL_EUNSUPPORTED, "Unsupported attention shape: " + std::to_string(c.heads) + " heads of " +
                                  std::to_string(c.head_dim) + " over " + std::to_string(c.kv_heads) + " KV heads.");
    const GgufTensor* embd = g.find("token_embd.weight");
    if (!embd) WL_THROW(WL_EUNSUPPORTED, "The model has no token_embd.weight.");
    c.vocab = embd->rows();
    return c;
}

static Weight weight_of(const GgufTensor& t)
{
    Weight w;
    w.type = t.type;
    w.cols = t.cols();
    w.experts = t.experts();
    const int64_t rows_all = t.elements() / t.dims[0];
    w.rows = (int)(rows_all / w.experts);
    w.row_bytes = t.size / rows_all;
    w.bytes = t.size;
    return w;
}

void Model::load_from_gguf(const Gguf& g)
{
    // Validate the layer tensors the forward indexes (ModelConfig.From, src/ModelConfig.cs:113-155).
    static const char* required[] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm"};
    static const char* olmo2[] = {"attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm", "attn_k_norm", "post_attention_norm", "post_ffw_norm"};
    for (int l = 0; l < c_.layers; ++l) {
        if (c_.post_norms) {
            for (const char* n : olmo2) if (!g.find(layer_name(l, n) + ".weight")) WL_THROW(WL_EUNSUPPORTED, "Layer " + std::to_string(l) + " has no " + n + ".weight (unsupported layout).");
        } else {
            for (const char* n : required) if (!g.find(layer_name(l, n) + ".weight")) WL_THROW(WL_EUNSUPPORTED, "Layer " + std::to_string(l) + " has no " + n + ".weight (unsupported layout).");
        }
        const bool moe = c_.expert_count > 0 && g.find(layer_name(l, "ffn_gate_inp.weight"));
        static const char* moe_names[] = {"ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"};
        static const char* dense_names[] = {"ffn_gate", "ffn_up", "ffn_down", "ffn_down"};
        const char* const* names = moe ? moe_names : dense_names;
        for (int i = 0; i < 4; ++i)
            if (!g.find(layer_name(l, names[i]) + ".weight"))
                WL_THROW(WL_EUNSUPPORTED, "Layer " + std::to_string(l) + " has no " + names[i] + ".weight (unsupported layout" +
                                          (moe ? "; Windlass reads the stacked expert tensors, not per-expert ffn_gate.N.weight files" : "") + ").");
        if (moe) {
            const GgufTensor* router = g.find(layer_name(l, "ffn_gate_inp.weight"));
            const GgufTensor* gate = g.find(layer_name(l, "ffn_gate_exps.weight"));
            const GgufTensor* up = g.find(layer_name(l, "ffn_up_exps.weight"));
            const GgufTensor* down = g.find(layer_name(l, "ffn_down_exps.weight"));
            if (router->cols() != c_.embd || router->rows() != c_.expert_count)
                WL_THROW(WL_EUNSUPPORTED, "Layer " + std::to_string(l) + ": ffn_gate_inp.weight has the wrong shape.");
            if (gate->ndims != 3 || gate->dims[2] != c_.expert_count || gate->cols() != c_.embd || up->ndims != 3 ||
                up->dims[2] != c_.expert_count || up->cols() != c_.embd || up->dims[1] != gate->dims[1])
                WL_THROW(WL_EUNSUPPORTED, "Layer " + std::to_string(l) + ": ffn_gate_exps/ffn_up_exps have the wrong shape.");
            if (down->ndims != 3 || down->dims[2] != c_.expert_count || down->dims[1] != c_.embd || down->dims[0] != gate->dims[1])
                WL_THROW(WL_EUNSUPPORTED, "Layer " + std::to_string(l) + ": ffn_down_exps has the wrong shape.");
            c_.expert_ff = (int)gate->dims[1];
        }
    }
    if (c_.qk_norm_full)        // the whole-vector QK norm (src/ModelConfig.cs:102-105)
        for (int l = 0; l < c_.layers; ++l) {
            const GgufTensor* qn = g.find(layer_name(l, "attn_q_norm.weight"));
            const GgufTensor* kn = g.find(layer_name(l, "attn_k_norm.weight"));
            if (!qn || !kn || qn->elements() != c_.qdim() || kn->elements() != c_.kvdim())
                WL_THROW(WL_EUNSUPPORTED, "Layer " + std::to_string(l) + ": attn_q_norm/attn_k_norm must cover the whole Q and K vectors (" +
                                          std::to_string(c_.qdim()) + " and " + std::to_string(c_.kvdim()) + ").");
        }
    for (const GgufTensor& t : g.tensors()) {
        const std::string& n = t.name;
        if (n.size() > 7 && n.compare(n.size() - 7, 7, ".weight") == 0 && t.ndims >= 2 && !can_decode(t.type))
            WL_THROW(WL_EUNSUPPORTED, "Tensor " + n + " uses " + type_name(t.type) + ", which Windlass cannot decode yet.");
    }

    // One arena for every tensor (this rank's part of it under tensor parallelism) plus the fp32 copies of the
    // vectors.
    const int G = tp_size_;
    int64_t total = 0;
    std::vector<int64_t> raw_upper((size_t)c_.layers + 1, 0), slot_upper((size_t)c_.layers + 1, 0);
    for (const GgufTensor& t : g.tensors()) {
        const int64_t bytes = G > 1 ? t.size / G + t.size / std::max<int64_t>(t.dims[1], 1) + 256 : t.size;
        const int st = t.ndims >= 2 ? stage_of_name(t.name) : -1;
        if (streamed_ && st >= 0 && st <= c_.layers) {
            // streamed matrices: bounded by their whole size, raw and in tiles (rows rounded up to 16)
            const int64_t rows_all = t.elements() / std::max<int64_t>(t.dims[0], 1);
            raw_upper[(size_t)st] += (t.size + 255) / 256 * 256;
            int64_t laid = ((rows_all + 15) / 16 * 16) * (t.size / std::max<int64_t>(rows_all, 1));
            if (k::tiles_supported(t.type, t.cols())) laid = std::max(laid, k::tile_bytes(t.type, (int)rows_all, t.cols()));
            slot_upper[(size_t)st] += laid + 256;
            continue;
        }
        total += (bytes + 255) / 256 * 256 + (t.elements() * 4 / (G > 1 ? G : 1) + 255) / 256 * 256;
    }
    if (G > 1 && c_.tied) if (const GgufTensor* t = g.find("token_embd.weight")) {
        const int64_t b = t->size / G + t->size / t->dims[1] + 512;
        if (streamed_) { raw_upper.back() += b; slot_upper.back() += (t->dims[1] + 15) / 16 * 16 * (t->size / t->dims[1]) / G + 512; }
        else total += b;
    }
    arena_ = dalloc<uint8_t>(total);
    arena_size_ = total;
    if (streamed_) plan_streaming(raw_upper, slot_upper);

    // split: WHOLE on every rank; ROWS this rank's 1/G of the rows; COLS its 1/G of every row's blocks; HEAD rows
    // rank*vocab_part_ .. +vocab_part_ (the last rank's may be fewer); EXPERTS a stacked tensor's experts
    // e_lo_ .. e_lo_ + e_n_ - 1, whole.
    enum Split { WHOLE, ROWS, COLS, HEAD, EXPERTS };
    auto upload = [&](const GgufTensor* t, Split sp) -> Weight {
        if (!t) return Weight{};
        Weight w = weight_of(*t);
        const uint8_t* src = g.data(*t);
        if (G == 1 || sp == WHOLE) {
            w.d = weight_alloc(w.bytes);
            WL_CUDA(cudaMemcpy(w.d, src, (size_t)w.bytes, cudaMemcpyHostToDevice));
            if (stream_file_ && cur_stage_ >= 0) file_src_.push_back({(int64_t)(w.d - staging_), {t->offset, t->size}});
        } else if (sp == EXPERTS) {
            if (w.experts != c_.expert_count || w.experts % G)
                WL_THROW(WL_EUNSUPPORTED, t->name + ": its experts do not split over " + std::to_string(G) + " GPUs.");
            const int64_t per = (int64_t)w.rows * w.row_bytes;
            w.experts = e_n_;
            w.bytes = per * e_n_;
            w.d = weight_alloc(w.bytes);
            WL_CUDA(cudaMemcpy(w.d, src + (int64_t)e_lo_ * per, (size_t)w.bytes, cudaMemcpyHostToDevice));
        } else if (sp == ROWS || sp == HEAD) {
            if (w.experts != 1) WL_THROW(WL_EUNSUPPORTED, "Tensor parallelism does not split stacked tensors.");
            int r0, n;
            if (sp == HEAD) { r0 = tp_rank_ * vocab_part_; n = std::min(vocab_part_, w.rows - r0); }
            else {
                if (w.rows % G) WL_THROW(WL_EUNSUPPORTED, t->name + ": " + std::to_string(w.rows) + " rows do not split over " + std::to_string(G) + " GPUs.");
                n = w.rows / G; r0 = tp_rank_ * n;
            }
            w.rows = n;
            w.bytes = (int64_t)n * w.row_bytes;
            w.d = weight_alloc(w.bytes);
            WL_CUDA(cudaMemcpy(w.d, src + (int64_t)r0 * w.row_bytes, (size_t)w.bytes, cudaMemcpyHostToDevice));
        } else {
            int b = 0, bb = 0;
            layout(w.type, &b, &bb);
            if (w.experts != 1 || w.cols % (G * b))
                WL_THROW(WL_EUNSUPPORTED, t->name + ": " + std::to_string(w.cols) + " columns do not split into whole " +
                                          type_name(w.type) + " blocks over " + std::to_string(G) + " GPUs.");
            const int64_t lrb = w.row_bytes / G;
            w.d = weight_alloc(lrb * w.rows);
            WL_CUDA(cudaMemcpy2D(w.d, (size_t)lrb, src + tp_rank_ * lrb, (size_t)w.row_bytes, (size_t)lrb, (size_t)w.rows,
                                 cudaMemcpyHostToDevice));
            w.cols /= G;
            w.row_bytes = lrb;
            w.bytes = lrb * w.rows;
        }
        stats_.bytes_h2d += w.bytes;
        weight_bytes_ += w.bytes;
        return w;
    };
    auto vec = [&](const GgufTensor* t, Split sp) -> Vec {
        Vec v;
        if (!t) return v;
        const uint8_t* src = g.data(*t);
        int64_t n = t->elements(), bytes = t->size;
        if (sp != WHOLE && G > 1) {      // a vector's split is a slice of its values (biases of split rows)
            if (t->type != 0 && t->type != 1)
                WL_THROW(WL_EUNSUPPORTED, t->name + " is not F32 or F16 and cannot be split over GPUs.");
            if (n % G) WL_THROW(WL_EUNSUPPORTED, t->name + " does not split over " + std::to_string(G) + " GPUs.");
            const int64_t esz = t->type == 0 ? 4 : 2;
            n /= G;
            src += tp_rank_ * n * esz;
            bytes = n * esz;
        }
        uint8_t* d = arena_alloc(bytes);
        WL_CUDA(cudaMemcpy(d, src, (size_t)bytes, cudaMemcpyHostToDevice));
        stats_.bytes_h2d += bytes;
        weight_bytes_ += bytes;
        v.n = (int)n;
        if (t->type == 0) v.d = (float*)d;
        else {
            v.d = (float*)arena_alloc(n * 4);
            k::dequant(t->type, d, n, v.d, stream_);
        }
        return v;
    };
    L_.resize(c_.layers);
    for (int l = 0; l < c_.layers; ++l) {
        LayerW& L = L_[l];
        auto T = [&](const char* n) { return g.find(layer_name(l, n)); };
        cur_stage_ = l;
        L.attn_norm = vec(T("attn_norm.weight"), WHOLE);
        L.q = upload(T("attn_q.weight"), ROWS); L.k = upload(T("attn_k.weight"), ROWS); L.v = upload(T("attn_v.weight"), ROWS);
        L.qb = vec(T("attn_q.bias"), ROWS); L.kb = vec(T("attn_k.bias"), ROWS); L.vb = vec(T("attn_v.bias"), ROWS);
        L.q_norm = vec(T("attn_q_norm.weight"), WHOLE); L.k_norm = vec(T("attn_k_norm.weight"), WHOLE);
        L.o = upload(T("attn_output.weight"), COLS);
        L.post_attn_norm = vec(T("post_attention_norm.weight"), WHOLE);
        L.ffn_norm = vec(T("ffn_norm.weight"), WHOLE);
        L.post_ffw_norm = vec(T("post_ffw_norm.weight"), WHOLE);
        L.moe = c_.expert_count > 0 && T("ffn_gate_inp.weight");
        if (L.moe) {
            L.router = upload(T("ffn_gate_inp.weight"), WHOLE);
            L.gate_exps = upload(T("ffn_gate_exps.weight"), EXPERTS); L.up_exps = upload(T("ffn_up_exps.weight"), EXPERTS);
            L.down_exps = upload(T("ffn_down_exps.weight"), EXPERTS);
            L.sh_gate = upload(T("ffn_gate_shexp.weight"), WHOLE); L.sh_up = upload(T("ffn_up_shexp.weight"), WHOLE);
            L.sh_down = upload(T("ffn_down_shexp.weight"), WHOLE);
            L.sh_gate_inp = upload(T("ffn_gate_inp_shexp.weight"), WHOLE);
            if (L.sh_gate.present()) c_.shared_expert_ff = L.sh_gate.rows;
        } else {
            L.gate = upload(T("ffn_gate.weight"), ROWS); L.up = upload(T("ffn_up.weight"), ROWS);
            L.down = upload(T("ffn_down.weight"), COLS);
        }
        end_stage(l, {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down, &L.router, &L.gate_exps, &L.up_exps,
                      &L.down_exps, &L.sh_gate, &L.sh_up, &L.sh_down, &L.sh_gate_inp});
    }
    cur_stage_ = -1;
    embd_ = upload(g.find("token_embd.weight"), WHOLE);
    out_norm_ = vec(g.find("output_norm.weight"), WHOLE);
    if (!out_norm_.present()) WL_THROW(WL_EUNSUPPORTED, "The model has no output_norm.weight.");
    cur_stage_ = c_.layers;
    output_ = c_.tied ? (G > 1 ? upload(g.find("token_embd.weight"), HEAD) : embd_) : upload(g.find("output.weight"), HEAD);
    end_stage(c_.layers, (c_.tied && G == 1) ? std::vector<Weight*>{} : std::vector<Weight*>{&output_});
    finish_streaming();

    std::vector<float> rf;
    if (const GgufTensor* t = g.find("rope_freqs.weight")) {
        if (t->type != 0) WL_THROW(WL_EUNSUPPORTED, "rope_freqs.weight must be F32.");
        rf.resize((size_t)t->elements());
        memcpy(rf.data(), g.data(*t), rf.size() * 4);
    }
    build_rope_table(rf.empty() ? nullptr : rf.data(), (int)rf.size());
    WL_CUDA(cudaStreamSynchronize(stream_));
}

// RopeTable (src/Transformer.cs:399-416) for every position of the context, in double, stored as float pairs.
void Model::build_rope_table(const float* rope_freqs, int n_rope_freqs)
{
    const int n = c_.rope_dims;
    std::vector<float> t((size_t)max_context_ * n);
    const double theta_scale = std::pow((double)c_.rope_base, -2.0 / n);
    for (int pos = 0; pos < max_context_; ++pos) {
        double theta = pos * (double)c_.rope_freq_scale;
        for (int i = 0; i < n / 2; ++i) {
            const double th = (rope_freqs && i < n_rope_freqs) ? theta / rope_freqs[i] : theta;
            t[(size_t)pos * n + 2 * i] = (float)std::cos(th);
            t[(size_t)pos * n + 2 * i + 1] = (float)std::sin(th);
            theta *= theta_scale;
        }
    }
    rope_table_ = dalloc<float>((int64_t)t.size());
    WL_CUDA(cudaMemcpy(rope_table_, t.data(), t.size() * 4, cudaMemcpyHostToDevice));
}

Model* Model::open_file(const std::string& path, const wl_options& opt)
{
    // The file and its shape are checked before any device work, so a bad file fails the same way with or without
    // a GPU.
    Gguf g(path);
    const Config c = read_config(g);
    check_tp(c, opt);
    std::unique_ptr<Model> m(new Model());
    m->c_ = c;
    m->file_path_ = path;
    m->init_device(opt);
    m->max_context_ = opt.max_context > 0 ? opt.max_context : std::min(m->c_.context_length, 8192);
    m->init_tp(opt);
    m->load_from_gguf(g);
    m->finish_open();
    return m.release();
}

// Synthetic models: tensor ids are (layer+1)<<8 | slot for layer tensors and 1..3 for the embedding, final norm and
// output head; the test oracle uses the same ids to regenerate any tensor on the CPU.
enum Slot { S_ATTN_NORM = 1, S_Q, S_K, S_V, S_O, S_FFN_NORM, S_GATE, S_UP, S_DOWN, S_Q_NORM, S_K_NORM, S_ROUTER,
            S_GATE_EXPS, S_UP_EXPS, S_DOWN_EXPS };

Model* Model::open_synthetic(const wl_synth_spec& sp, const wl_options& opt)
{
    if (opt.stream_file != 0) WL_THROW(WL_EINVAL, "stream_file reads the layers from a GGUF file; a synthetic model has none.");
    std::unique_ptr<Model> m(new Model());
    Config& c = m->c_;
    c.arch = std::string(sp.arch, strnlen(sp.arch, sizeof sp.arch));
    if (c.arch != "llama" && c.arch != "qwen3" && c.arch != "qwen3moe") WL_THROW(WL_EUNSUPPORTED, "synthetic arch must be llama, qwen3 or qwen3moe");
    c.layers = sp.layers; c.embd = sp.embd; c.heads = sp.heads; c.kv_heads = sp.kv_heads;
    c.head_dim = sp.head_dim > 0 ? sp.head_dim : sp.embd / std::max(1, sp.heads);
    c.rope_dims = c.head_dim; c.vocab = sp.vocab; c.context_length = sp.context_length > 0 ? sp.context_length : 4096;
    c.rms_eps = sp.rms_eps > 0 ? sp.rms_eps : 1e-5f; c.rope_base = sp.rope_base > 0 ? sp.rope_base : 10000.f;
    c.rope_neox = c.arch != "llama";
    c.qk_norm = c.arch != "llama";
    if (c.arch == "qwen3moe") {
        c.expert_count = sp.experts; c.expert_used = sp.experts_used; c.expert_ff = sp.expert_ff; c.expert_weights_norm = true;
        if (c.expert_count < 1 || c.expert_count > 256 || c.expert_used < 1 || c.expert_used > c.expert_count)
            WL_THROW(WL_EINVAL, "bad synthetic expert counts");
    }
    if (c.layers <= 0 || c.embd <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads || c.vocab <= 0)
        WL_THROW(WL_EINVAL, "bad synthetic shape");
    check_tp(c, opt);
    m->init_device(opt);
    m->max_context_ = opt.max_context > 0 ? opt.max_context : std::min(c.context_length, 8192);
    const float sigma = sp.sigma > 0 ? sp.sigma : 0.02f;
    const int QD = c.qdim(), KD = c.kvdim(), E = c.embd, F = sp.ff, NE = c.expert_count, X = c.expert_ff;
    m->init_tp(opt);
    const int G = m->tp_size_, rank = m->tp_rank_;

    // split (tensor parallelism): 0 whole, 1 rows, 2 columns, 3 output-head rows; the full tensor is generated and
    // this rank's part copied out, so every rank holds exactly the bytes of the one-GPU model's slice.
    struct Plan { Weight* w; Vec* v; uint32_t tid; int type; int64_t rows, cols; int experts; int split = 0; };
    std::vector<Plan> plan;
    m->L_.resize(c.layers);
    for (int l = 0; l < c.layers; ++l) {
        LayerW& L = m->L_[l];
        const uint32_t b = (uint32_t)(l + 1) << 8;
        plan.push_back({nullptr, &L.attn_norm, b | S_ATTN_NORM, 0, 1, E, 1});
        plan.push_back({&L.q, nullptr, b | S_Q, sp.type_attn, QD, E, 1, 1});
        plan.push_back({&L.k, nullptr, b | S_K, sp.type_attn, KD, E, 1, 1});
        plan.push_back({&L.v, nullptr, b | S_V, sp.type_attn_v, KD, E, 1, 1});
        if (c.qk_norm) {
            plan.push_back({nullptr, &L.q_norm, b | S_Q_NORM, 0, 1, c.head_dim, 1});
            plan.push_back({nullptr, &L.k_norm, b | S_K_NORM, 0, 1, c.head_dim, 1});
        }
        plan.push_back({&L.o, nullptr, b | S_O, sp.type_attn, E, QD, 1, 2});
        plan.push_back({nullptr, &L.ffn_norm, b | S_FFN_NORM, 0, 1, E, 1});
        if (NE > 0) {
            L.moe = true;
            plan.push_back({&L.router, nullptr, b | S_ROUTER, 0, NE, E, 1});
            // under tensor parallelism rank r keeps experts r*NE/G .., which are contiguous rows of the stack
            plan.push_back({&L.gate_exps, nullptr, b | S_GATE_EXPS, sp.type_ffn, (int64_t)NE * X, E, NE, 1});
            plan.push_back({&L.up_exps, nullptr, b | S_UP_EXPS, sp.type_ffn, (int64_t)NE * X, E, NE, 1});
            plan.push_back({&L.down_exps, nullptr, b | S_DOWN_EXPS, sp.type_ffn_down, (int64_t)NE * E, X, NE, 1});
        } else {
            plan.push_back({&L.gate, nullptr, b | S_GATE, sp.type_ffn, F, E, 1, 1});
            plan.push_back({&L.up, nullptr, b | S_UP, sp.type_ffn, F, E, 1, 1});
            plan.push_back({&L.down, nullptr, b | S_DOWN, sp.type_ffn_down, E, F, 1, 2});
        }
    }
    plan.push_back({&m->embd_, nullptr, 1, sp.type_embd, c.vocab, E, 1});
    plan.push_back({nullptr, &m->out_norm_, 2, 0, 1, E, 1});
    plan.push_back({&m->output_, nullptr, 3, sp.type_output, c.vocab, E, 1, 3});

    // this rank's rows [r0, r0 + nrows) and column blocks [c0, c0 + ncols) of a planned tensor
    auto part = [&](const Plan& p, int64_t* r0, int64_t* nrows, int64_t* c0, int64_t* ncols) {
        *r0 = 0; *nrows = p.rows; *c0 = 0; *ncols = p.cols;
        if (G == 1 || p.split == 0) return;
        const int blk = p.type == 0 ? 1 : p.type == 8 ? 32 : 256;
        if (p.split == 1) {
            if (p.rows % G) WL_THROW(WL_EUNSUPPORTED, "synthetic tensor rows do not split over " + std::to_string(G) + " GPUs");
            *nrows = p.rows / G; *r0 = rank * *nrows;
        } else if (p.split == 3) {
            *r0 = (int64_t)rank * m->vocab_part_; *nrows = std::min<int64_t>(m->vocab_part_, p.rows - *r0);
        } else {
            if (p.cols % ((int64_t)G * blk))
                WL_THROW(WL_EUNSUPPORTED, "synthetic tensor columns do not split into whole blocks over " + std::to_string(G) + " GPUs");
            *ncols = p.cols / G; *c0 = rank * *ncols;
        }
    };
    // the stage of a planned tensor under streaming: matrices of layer l stream with stage l, the output head with
    // the head stage; the embedding and every vector stay resident
    auto stage_of = [&](const Plan& p) -> int {
        if (!m->streamed_ || p.v) return -1;
        if (p.tid >= 256) return (int)(p.tid >> 8) - 1;
        return p.tid == 3 ? c.layers : -1;
    };
    int64_t total = 0, tmp_bytes = 0;
    std::vector<int64_t> raw_upper((size_t)c.layers + 1, 0), slot_upper((size_t)c.layers + 1, 0);
    for (const Plan& p : plan) {
        const int64_t rb = row_bytes_of(p.type, p.cols);
        if (rb <= 0 || p.cols % (p.type == 0 ? 1 : p.type == 8 ? 32 : 256) != 0) WL_THROW(WL_EUNSUPPORTED, "synthetic tensor shape does not fit its type");
        int64_t r0, nr, c0, nc;
        part(p, &r0, &nr, &c0, &nc);
        const int64_t bytes = (row_bytes_of(p.type, nc) * nr + 255) / 256 * 256;
        const int st = stage_of(p);
        if (st >= 0) {
            raw_upper[(size_t)st] += bytes;
            int64_t laid = (nr + 15) / 16 * 16 * row_bytes_of(p.type, nc);
            if (k::tiles_supported(p.type, (int)nc)) laid = std::max(laid, k::tile_bytes(p.type, (int)nr, (int)nc));
            slot_upper[(size_t)st] += laid + 256;
        } else {
            total += bytes;
        }
        if (G > 1 && p.split) tmp_bytes = std::max(tmp_bytes, rb * p.rows);
    }
    m->arena_ = dalloc<uint8_t>(total);
    m->arena_size_ = total;
    if (m->streamed_) m->plan_streaming(raw_upper, slot_upper);
    std::vector<Weight*> stage_ws;
    uint8_t* tmp = tmp_bytes ? dalloc<uint8_t>(tmp_bytes) : nullptr;
    try {
        for (const Plan& p : plan) {
            int64_t r0, nr, c0, nc;
            part(p, &r0, &nr, &c0, &nc);
            const bool is_vec = p.v != nullptr;
            const int st = stage_of(p);
            // a matrix of another stage (or a resident one) completes the stage being loaded; vectors are always
            // resident and leave it open
            if (!is_vec && st != m->cur_stage_) {
                if (m->cur_stage_ >= 0) m->end_stage(m->cur_stage_, stage_ws);
                stage_ws.clear();
                m->cur_stage_ = st;
            }
            const int64_t full_rb = row_bytes_of(p.type, p.cols);
            Weight w;
            w.type = p.type; w.cols = (int)nc;
            w.experts = G > 1 && p.split == 1 && p.experts > 1 ? p.experts / G : p.experts;
            w.rows = (int)(nr / w.experts);
            w.row_bytes = row_bytes_of(p.type, nc); w.bytes = w.row_bytes * nr;
            w.d = is_vec ? m->arena_alloc(w.bytes) : m->weight_alloc(w.bytes);
            if (G == 1 || p.split == 0) {
                k::synth(p.type, sp.seed, p.tid, p.rows, p.cols, sigma, is_vec ? 1.0f : 0.0f, w.d, m->stream_);
            } else {
                k::synth(p.type, sp.seed, p.tid, p.rows, p.cols, sigma, 0.0f, tmp, m->stream_);
                const int64_t cb = row_bytes_of(p.type, c0);    // byte offset of the first column block
                WL_CUDA(cudaMemcpy2DAsync(w.d, (size_t)w.row_bytes, tmp + r0 * full_rb + cb, (size_t)full_rb,
                                          (size_t)w.row_bytes, (size_t)nr, cudaMemcpyDeviceToDevice, m->stream_));
            }
            m->weight_bytes_ += w.bytes;
            if (is_vec) { p.v->d = (float*)w.d; p.v->n = (int)(nr * nc); }
            else *p.w = w;
            if (st >= 0) stage_ws.push_back(p.w);
        }
        if (m->cur_stage_ >= 0) m->end_stage(m->cur_stage_, stage_ws);
        m->finish_streaming();
        WL_CUDA(cudaStreamSynchronize(m->stream_));
    } catch (...) {
        if (tmp) cudaFree(tmp);
        throw;
    }
    if (tmp) cudaFree(tmp);
    m->build_rope_table(nullptr, 0);
    WL_CUDA(cudaStreamSynchronize(m->stream_));
    m->finish_open();
    return m.release();
}

void Model::finish_open()
{
    if (!k::attention_supported(c_.heads, c_.kv_heads, c_.head_dim))
        WL_THROW(WL_EUNSUPPORTED, "Unsupported attention shape: " + std::to_string(c_.heads) + " heads of " +
                                  std::to_string(c_.head_dim) + " over " + std::to_string(c_.kv_heads) + " KV heads.");
    if (!rope_table_) build_rope_table(nullptr, 0);
    build_maps();
    own_ = new_seq();
    opened_ = true;
}

Model::~Model()
{
    if (device_ >= 0) cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    if (side_) cudaStreamSynchronize(side_);
    drop_graphs();
    if (own_) free_seq(own_);
    dfree(arena_); dfree(rope_table_);
    dfree(x_); dfree(xn_); dfree(q_); dfree(k_); dfree(v_); dfree(att_); dfree(o_); dfree(g_); dfree(u_);
    dfree(logits_); dfree(router_); dfree(wts_); dfree(xe_); dfree(ye_); dfree(ge_); dfree(ue_); dfree(moe_out_);
    dfree(sh_gl_); dfree(tok_d_); dfree(pos_d_); dfree(sel_); dfree(bad_d_); dfree(etok_d_); dfree(ew_d_); dfree(rows_d_);
    hfree(h_tok_); hfree(h_pos_); hfree(h_rows_); hfree(h_sel_); hfree(h_wts_); hfree(h_etok_); hfree(h_ew_);
    for (void* p : extra_allocs_) cudaFree(p);
    if (xprep_buf_) cudaFree(xprep_buf_);
    if (gemm_buf_) cudaFree(gemm_buf_);
    dfree(att_part_);
    dfree(err_d_);
    if (comm_) {
        try { close_fused_ar(); } catch (...) {}
    }
    free_streaming();
    dfree(logits_part_); dfree(logits_all_); dfree(flag_d_); hfree(flag_h_);
    dfree(pg_); dfree(pu_); dfree(py_); dfree(expert_count_d_);
    dfree(ids_d_); dfree(amax_key_); dfree(amax_count_); dfree(gen_d_); hfree(h_ids_); hfree(h_gen_);
    dfree(sample_ws_);
    if (pprep_) cudaFree(pprep_);
    comm_.reset();           // after the graphs that hold its collectives
    for (const ProfileMark& m : marks_) { cudaEventDestroy(m.start); cudaEventDestroy(m.stop); }
    for (cudaEvent_t e : event_pool_) cudaEventDestroy(e);
    if (fork_ev_) cudaEventDestroy(fork_ev_);
    if (join_ev_) cudaEventDestroy(join_ev_);
    if (side_) cudaStreamDestroy(side_);
    if (stream_) cudaStreamDestroy(stream_);
}

int64_t Model::device_bytes() const
{
    return arena_size_ + (int64_t)max_context_ * c_.rope_dims * 4;
}

// ---------------------------------------------------------------------------------------------------------------------
// sequences
// ---------------------------------------------------------------------------------------------------------------------
Seq* Model::new_seq()
{
    Seq* s = new Seq();
    s->model = this;
    return s;
}

void Model::free_seq(Seq* s)
{
    if (!s) return;
    WL_CUDA(cudaSetDevice(device_));
    WL_CUDA(cudaStreamSynchronize(stream_));
    if (s->kv) cudaFree(s->kv);
    delete s;
}

// Transformer.Reserve (src/Transformer.cs:62-73): grow to max(positions, min(context, max(256, 2*capacity))).
void Model::reserve(Seq* s, int positions)
{
    if (positions <= s->capacity) return;
    const int cap = std::max(positions, std::min(max_context_, std::max(256, s->capacity * 2)));
    const int64_t KD = c_.kvdim(), per_layer = (int64_t)cap * KD;
    uint16_t* nk = dalloc<uint16_t>(2 * (int64_t)c_.layers * per_layer);
    if (s->kv && s->length > 0) {
        const int64_t old_per_layer = (int64_t)s->capacity * KD;
        // rows = 2*layers blocks of `length` positions
        WL_CUDA(cudaMemcpy2DAsync(nk, per_layer * 2, s->kv, old_per_layer * 2, (size_t)s->length * KD * 2, 2 * c_.layers,
                                  cudaMemcpyDeviceToDevice, stream_));
    }
    WL_CUDA(cudaStreamSynchronize(stream_));
    if (s->kv) cudaFree(s->kv);
    s->kv = nk;
    s->capacity = cap;
}

// ---------------------------------------------------------------------------------------------------------------------
// workspaces
// ---------------------------------------------------------------------------------------------------------------------
void Model::ensure_workspace(int T, int logit_rows)
{
    const int E = c_.embd, QD = c_.qdim(), KD = c_.kvdim();
    int F = 0;
    for (const LayerW& L : L_) {
        if (L.gate.present()) F = std::max(F, L.gate.rows);
        if (L.sh_gate.present()) F = std::max(F, L.sh_gate.rows);
    }
    if (T > ws_T_) {
        const int n = std::max(T, ws_T_ * 2 > 0 ? std::min(ws_T_ * 2, std::max(T, 8)) : T);
        dfree(x_); dfree(xn_); dfree(q_); dfree(k_); dfree(v_); dfree(att_); dfree(o_); dfree(g_); dfree(u_);
        dfree(router_); dfree(wts_); dfree(xe_); dfree(ye_); dfree(ge_); dfree(ue_); dfree(moe_out_); dfree(sh_gl_);
        dfree(tok_d_); dfree(pos_d_); dfree(sel_); dfree(bad_d_); dfree(etok_d_); dfree(ew_d_); dfree(rows_d_);
        x_ = dalloc<float>((int64_t)n * E); xn_ = dalloc<float>((int64_t)n * E); o_ = dalloc<float>((int64_t)n * E);
        q_ = dalloc<float>((int64_t)n * QD); att_ = dalloc<float>((int64_t)n * QD);
        k_ = dalloc<float>((int64_t)n * KD); v_ = dalloc<float>((int64_t)n * KD);
        g_ = dalloc<float>((int64_t)n * std::max(F, 1)); u_ = dalloc<float>((int64_t)n * std::max(F, 1));
        tok_d_ = dalloc<int32_t>(n); pos_d_ = dalloc<int32_t>(n); bad_d_ = dalloc<int32_t>(1);
        rows_d_ = dalloc<RowKV>(n);
        if (c_.expert_count > 0) {
            const int NE = c_.expert_count, K = c_.expert_used, X = std::max(c_.expert_ff, 1);
            router_ = dalloc<float>((int64_t)n * NE); wts_ = dalloc<float>((int64_t)n * K); sel_ = dalloc<int32_t>((int64_t)n * K);
            xe_ = dalloc<float>((int64_t)n * E); ye_ = dalloc<float>((int64_t)n * E); moe_out_ = dalloc<float>((int64_t)n * E);
            ge_ = dalloc<float>((int64_t)n * X); ue_ = dalloc<float>((int64_t)n * X); sh_gl_ = dalloc<float>(n);
            etok_d_ = dalloc<int32_t>((int64_t)n * K); ew_d_ = dalloc<float>((int64_t)n * K);
        }
        hfree(h_tok_); hfree(h_pos_); hfree(h_rows_); hfree(h_sel_); hfree(h_wts_); hfree(h_etok_); hfree(h_ew_);
        h_tok_ = halloc<int32_t>(n); h_pos_ = halloc<int32_t>(n); h_rows_ = halloc<RowKV>(n);
        if (c_.expert_count > 0) {
            const int K = c_.expert_used;
            h_sel_ = halloc<int32_t>((int64_t)n * K); h_wts_ = halloc<float>((int64_t)n * K);
            h_etok_ = halloc<int32_t>((int64_t)n * K); h_ew_ = halloc<float>((int64_t)n * K);
        }
        ws_T_ = n;
        ws_gen_++;
        drop_graphs();
    }
    if (!xprep_buf_) {
        int max_cols = c_.embd;
        for (const LayerW& L : L_) {
            for (const Weight* w : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down, &L.gate_exps, &L.up_exps,
                                    &L.down_exps, &L.sh_gate, &L.sh_up, &L.sh_down})
                if (w->present()) max_cols = std::max(max_cols, w->cols);
        }
        WL_CUDA(cudaMalloc(&xprep_buf_, k::xprep_bytes(max_cols, 8)));
        const size_t apf = k::attention_part_floats(c_.heads, c_.kv_heads, c_.head_dim);
        att_part_ = dalloc<float>((int64_t)apf);
        WL_CUDA(cudaMemset(att_part_, 0, sizeof(float) * apf));     // the merge tickets start at zero
    }
    if (logit_rows > ws_logit_rows_) {
        dfree(logits_); dfree(ids_d_); dfree(amax_key_); dfree(amax_count_); hfree(h_ids_);
        logits_ = dalloc<float>((int64_t)logit_rows * c_.vocab);
        ids_d_ = dalloc<int32_t>(logit_rows);
        amax_key_ = dalloc<unsigned long long>(logit_rows);
        amax_count_ = dalloc<unsigned>(logit_rows);
        WL_CUDA(cudaMemset(amax_key_, 0, sizeof(unsigned long long) * (size_t)logit_rows));
        WL_CUDA(cudaMemset(amax_count_, 0, sizeof(unsigned) * (size_t)logit_rows));
        h_ids_ = halloc<int32_t>(logit_rows);
        if (tp_size_ > 1) {
            dfree(logits_part_); dfree(logits_all_);
            logits_part_ = dalloc<float>((int64_t)logit_rows * vocab_part_);
            logits_all_ = dalloc<float>((int64_t)tp_size_ * logit_rows * vocab_part_);
        }
        ws_logit_rows_ = logit_rows;
        ws_gen_++;
        drop_graphs();
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------------------------------------
// y[T][rows] = W x. Formats with a tensor-core matvec take activations prepared by k::xprep (8 columns at a time);
// reuse_x says x is the input of the previous matmul as well, so its prepared form can be reused.
void Model::matmul(const Weight& w, const float* x, int T, float* y, int path, bool reuse_x, int64_t ldy)
{
    if (ldy <= 0) ldy = w.rows;
    // path 1 (or prefill_path 1 for prompts): the fp32 CUDA-core kernel
    const bool cuda_cores = path == 1 || (T > 8 && prefill_path_ == 1);
    // more than 8 rows of Q4_K: the tcgen05 GEMM (prefill_path 2 keeps the integer matvec in 8-column chunks)
    if (!cuda_cores && T >= k::gemm_min_rows(w.type) && prefill_path_ != 2 && !each_token_ && w.tiles &&
        w.row_base % 16 == 0 && k::gemm_supported(w.type, w.cols)) {
        const size_t need = k::gemm_scratch_bytes(T, w.cols);
        if (need > gemm_buf_bytes_) {
            WL_CUDA(cudaStreamSynchronize(stream_));
            if (gemm_buf_) cudaFree(gemm_buf_);
            gemm_buf_ = nullptr;
            gemm_buf_bytes_ = 0;
            WL_CUDA(cudaMalloc(&gemm_buf_, need));
            gemm_buf_bytes_ = need;
        }
        prep_x_ = nullptr;
        const int mark = profile_begin();
        k::gemm_tiles(w.type, w.tiles, w.row_base, w.rows, w.cols, x, w.cols, T, y, ldy, gemm_buf_, err_d_, stream_);
        profile_end(mark, w.type, (double)w.rows * w.row_bytes + 4.0 * T * ((double)w.cols + w.rows));
        return;
    }
    if (!cuda_cores && w.tiles && w.row_base % 16 == 0 && xprep_buf_) {
        for (int c0 = 0; c0 < T; c0 += 8) {
            const int nc = std::min(8, T - c0);
            const k::XPrep p = k::xprep_view(xprep_buf_, w.cols, nc);
            const bool same = reuse_x && T <= 8 && prep_x_ == x && prep_cols_ == w.cols && prep_nc_ == nc;
            if (!same) {
                const int pm = profile_begin();
                k::xprep(x + (int64_t)c0 * w.cols, w.cols, w.cols, nc, p, stream_);
                profile_end(pm, WL_PROFILE_XPREP, 0.0);
                prep_x_ = x; prep_cols_ = w.cols; prep_nc_ = nc;
            }
            const int mark = profile_begin();
            const bool push = ar_out_ && w.type == 12 && T <= 8;
            k::matvec_tiles(w.type, w.tiles, w.row_base, w.rows, w.cols, p, y + (int64_t)c0 * ldy, ldy, err_d_,
                            stream_, push ? ar_out_ : nullptr);
            if (push) ar_out_done_ = true;
            profile_end(mark, w.type, (double)w.rows * w.row_bytes + 4.0 * nc * ((double)w.cols + w.rows));
        }
        if (T > 8) prep_x_ = nullptr;
        return;
    }
    prep_x_ = nullptr;
    if (w.streamed_tiles) WL_THROW(WL_EUNSUPPORTED, "a streamed weight holds tiles only and has no CUDA-core path");
    const int mark = profile_begin();
    k::matvec(w.type, w.d, w.row_bytes, w.rows, w.cols, x, w.cols, T, y, ldy, stream_);
    profile_end(mark, w.type, (double)w.rows * w.row_bytes + 4.0 * T * ((double)w.cols + w.rows));
}

void Model::matmul2(const Weight& a, const Weight& b, const float* x, int T, float* ya, float* yb)
{
    // one launch for both matrices at decode: the second matrix's CTAs follow the first's with no launch boundary
    // between them (measured on the 70B step: 4 us a layer less than two launches for gate and up)
    const bool pair = T <= 8 && a.present() && b.present() && a.type == 12 && b.type == 12 && a.tiles && b.tiles &&
                      a.cols == b.cols && a.row_base % 16 == 0 && b.row_base % 16 == 0 && xprep_buf_;
    if (!pair) {
        matmul(a, x, T, ya, 0, true);
        matmul(b, x, T, yb, 0, true);
        return;
    }
    const k::XPrep p = k::xprep_view(xprep_buf_, a.cols, T);
    if (!(prep_x_ == x && prep_cols_ == a.cols && prep_nc_ == T)) {
        const int pm = profile_begin();
        k::xprep(x, a.cols, a.cols, T, p, stream_);
        profile_end(pm, WL_PROFILE_XPREP, 0.0);
        prep_x_ = x; prep_cols_ = a.cols; prep_nc_ = T;
    }
    const int mark = profile_begin();
    k::matvec_tiles2(a.tiles, a.row_base, a.rows, ya, a.rows, b.tiles, b.row_base, b.rows, yb, b.rows, a.cols, p, err_d_,
                     stream_);
    profile_end(mark, a.type, (double)a.rows * a.row_bytes + (double)b.rows * b.row_bytes +
                                  4.0 * T * ((double)a.cols + a.rows + b.rows));
}

// Starts a profiled region (an event pair around launches on the model's stream); -1 when profiling is off.
int Model::profile_begin()
{
    if (!profiling_) return -1;
    while (event_pool_.size() < 2) {
        cudaEvent_t e;
        WL_CUDA(cudaEventCreate(&e));
        event_pool_.push_back(e);
    }
    ProfileMark m{};
    m.start = event_pool_.back(); event_pool_.pop_back();
    m.stop = event_pool_.back(); event_pool_.pop_back();
    WL_CUDA(cudaEventRecord(m.start, stream_));
    marks_.push_back(m);
    return (int)marks_.size() - 1;
}

void Model::profile_end(int mark, int kind, double bytes)
{
    if (mark < 0) return;
    ProfileMark& m = marks_[(size_t)mark];
    m.type = kind;
    m.bytes = bytes;
    WL_CUDA(cudaEventRecord(m.stop, stream_));
    if (marks_.size() > 4096) flush_profile();
}

static Weight slice(const Weight& w, int e)
{
    Weight s = w;
    s.d = const_cast<uint8_t*>(w.expert(e));
    s.experts = 1;
    s.bytes = (int64_t)w.rows * w.row_bytes;
    s.row_base = w.row_base + e * w.rows;
    return s;
}

// Tensor maps for every weight the tensor-core matvec can read.
void Model::build_maps()
{
    auto mk = [&](Weight& w) {
        // Q4_K / Q6_K, Q8_0, IQ4_XS, IQ2_XXS: a tile-major copy for the tensor-core matvec (expert slices must start
        // on a tile; only Q4_K and Q6_K experts are read from tiles)
        if (w.present() && !w.tiles && k::tiles_supported(w.type, w.cols) &&
            (w.experts == 1 || ((w.type == 12 || w.type == 14) && w.rows % 16 == 0))) {
            const int total = w.rows * w.experts;
            void* t = nullptr;
            WL_CUDA(cudaMalloc(&t, (size_t)k::tile_bytes(w.type, total, w.cols)));
            extra_allocs_.push_back(t);
            w.tiles = (uint8_t*)t;
            k::make_tiles(w.type, w.d, total, w.cols, w.row_bytes, w.tiles, stream_);
        }
    };
    for (LayerW& L : L_)
        for (Weight* w : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down, &L.router, &L.gate_exps, &L.up_exps,
                          &L.down_exps, &L.sh_gate, &L.sh_up, &L.sh_down, &L.sh_gate_inp})
            mk(*w);
    mk(output_);
    if (!err_d_) {
        err_d_ = dalloc<int>(1);
        WL_CUDA(cudaMemset(err_d_, 0, sizeof(int)));
    }
    if (c_.expert_count > 0 && !expert_count_d_) {
        // [0] the count, [1] where a graph capture keeps it while its warm-up run repeats a step
        expert_count_d_ = dalloc<unsigned long long>(2);
        WL_CUDA(cudaMemset(expert_count_d_, 0, 2 * sizeof(unsigned long long)));
    }
}

// A bounded device wait that gave up leaves a code in err_d_; report it once the stream is idle.
void Model::check_device_error()
{
    if (expert_count_d_) {
        unsigned long long n = 0;
        WL_CUDA(cudaMemcpy(&n, expert_count_d_, sizeof n, cudaMemcpyDeviceToHost));
        if (n) {
            stats_.expert_runs += (int64_t)n;
            WL_CUDA(cudaMemset(expert_count_d_, 0, sizeof n));
        }
    }
    int e = 0;
    WL_CUDA(cudaMemcpy(&e, err_d_, sizeof(int), cudaMemcpyDeviceToHost));
    if (e != 0) {
        WL_CUDA(cudaMemset(err_d_, 0, sizeof(int)));
        WL_THROW(WL_ETIMEDOUT, "a device-side wait gave up (code " + std::to_string(e) + ")");
    }
}

void Model::ffn_dense(const LayerW& L, int T)
{
    const int F = L.gate.rows;
    matmul2(L.gate, L.up, xn_, T, g_, u_);
    prep_x_ = nullptr;
    const int sm = profile_begin();
    if (L.down.tiles && T <= 8 && F % 256 == 0 && xprep_buf_) {
        const k::XPrep p = k::xprep_view(xprep_buf_, F, T);
        k::swiglu_prep(g_, u_, T, F, p, stream_);
        prep_x_ = g_; prep_cols_ = F; prep_nc_ = T;
    } else {
        k::swiglu(g_, u_, (int64_t)T * F, stream_);
    }
    profile_end(sm, WL_PROFILE_SWIGLU, 0.0);
    matmul_reduce(L.down, g_, T);
}

// Decode steps of a mixture-of-experts layer stay on the device when the experts are tiled Q4_K (whole 16-row tiles
// per expert) and there is no shared expert: the router's choice never goes to the host, so the step can also be a
// CUDA graph.
bool Model::moe_on_device(const LayerW& L, int T) const
{
    const Weight &g = L.gate_exps, &u = L.up_exps, &d = L.down_exps;
    return L.moe && T <= 8 && !L.sh_gate.present() && xprep_buf_ && g.tiles && u.tiles && d.tiles && g.type == 12 &&
           u.type == 12 && d.type == 12 && g.rows % 16 == 0 && d.rows % 16 == 0 && g.cols == c_.embd &&
           d.cols == g.rows && g.row_base == 0 && u.row_base == 0 && d.row_base == 0;
}

// MoeFfn on the device: router matvec, top-k (k_route), then one grouped matvec launch each for gate, up and down over
// every (token, chosen expert) pair, the experts' ids read on the device, and the weighted sum per token in
// ascending expert order, the order the reference adds them (src/Transformer.cs:280-293). Each pair's expert output
// is the bits the host path's per-expert matvec gives, so the result is too.
void Model::ffn_moe_device(const LayerW& L, int T)
{
    const int E = c_.embd, K = c_.expert_used, X = L.gate_exps.rows, NP = T * K;
    if (NP > pair_cap_) {
        WL_CUDA(cudaStreamSynchronize(stream_));
        dfree(pg_); dfree(pu_); dfree(py_);
        if (pprep_) cudaFree(pprep_);
        pprep_ = nullptr;
        const int cap = 8 * K;
        pg_ = dalloc<float>((int64_t)cap * X);
        pu_ = dalloc<float>((int64_t)cap * X);
        py_ = dalloc<float>((int64_t)cap * E);
        WL_CUDA(cudaMalloc(&pprep_, k::xprep_bytes(X, cap)));
        pair_cap_ = cap;
        ws_gen_++;
        drop_graphs();
    }
    const k::XPrep px = k::xprep_view(xprep_buf_, E, T);        // xn_, prepared by the ffn norm
    matmul(L.router, xn_, T, router_);
    k::route(router_, T, c_.expert_count, K, c_.expert_weights_norm ? 1 : 0, sel_, wts_, stream_,
             T == 1 ? expert_count_d_ : nullptr);
    if (T > 1) k::count_experts(sel_, NP, expert_count_d_, stream_);
    const int mark = profile_begin();
    // under tensor parallelism the pairs of experts held by other GPUs are skipped here (their rows of pg_, pu_ and
    // py_ are left as they are and never read)
    k::matvec_pairs2(L.gate_exps.tiles, L.up_exps.tiles, X, E, sel_, NP, K, px, pg_, pu_, X, err_d_, stream_, e_lo_,
                     e_n_);
    const k::XPrep pp = k::xprep_view(pprep_, X, NP);
    k::swiglu_prep(pg_, pu_, NP, X, pp, stream_);
    k::matvec_pairs(L.down_exps.tiles, 0, E, X, sel_, NP, K, false, pp, py_, E, err_d_, stream_, e_lo_, e_n_);
    profile_end(mark, 12, (double)NP * ((double)L.gate_exps.row_bytes * X * 2 + (double)L.down_exps.row_bytes * E));
    if (tp_size_ > 1) {
        // this GPU's experts' weighted sum, then the sum over the GPUs: fused into the next norm through this rank's
        // all-reduce slot (decode steps), else NCCL
        if (ar_on_ && T <= k::AR_COLS && ar_idx_ < k::AR_STEP) {
            const int idx = ar_idx_++;
            float* stage = reinterpret_cast<float*>(ar_buf_ + k::ar_slot_offset(idx, E));
            k::moe_combine(py_, sel_, wts_, T, K, E, stage, stream_, e_lo_, e_n_);
            k::ar_push(stage, T, ar_out(idx), stream_);
            pending_ar_ = idx;
        } else {
            k::moe_combine(py_, sel_, wts_, T, K, E, o_, stream_, e_lo_, e_n_);
            all_reduce(o_, (int64_t)T * E);
        }
    } else if (k::norm_prep_supported(E) && !c_.post_norms && K <= 16) {
        // the next norm (the next layer's or the head's) combines the experts' outputs as it adds the residual
        pending_moe_ = true;
        moe_in_ = k::MoeIn{py_, sel_, wts_, K};
    } else {
        k::moe_combine(py_, sel_, wts_, T, K, E, o_, stream_);
    }
    prep_x_ = nullptr;
}

// MoeFfn (src/Transformer.cs:259-311): router, top-k, then each chosen expert runs once on the rows routed to it, in
// expert order; the weighted outputs are added per row in that same order, so a row's result does not depend on the
// other rows of the step.
void Model::ffn_moe(const LayerW& L, int T)
{
    const int E = c_.embd, NE = c_.expert_count, K = c_.expert_used, X = L.gate_exps.rows;
    matmul(L.router, xn_, T, router_);
    k::route(router_, T, NE, K, c_.expert_weights_norm ? 1 : 0, sel_, wts_, stream_);
    WL_CUDA(cudaMemcpyAsync(h_sel_, sel_, sizeof(int32_t) * (size_t)T * K, cudaMemcpyDeviceToHost, stream_));
    WL_CUDA(cudaMemcpyAsync(h_wts_, wts_, sizeof(float) * (size_t)T * K, cudaMemcpyDeviceToHost, stream_));
    WL_CUDA(cudaStreamSynchronize(stream_));
    std::vector<int> count(NE, 0), start(NE + 1, 0);
    for (int i = 0; i < T * K; ++i) count[h_sel_[i]]++;
    for (int e = 0; e < NE; ++e) start[e + 1] = start[e] + count[e];
    std::vector<int> at(start.begin(), start.end() - 1);
    for (int t = 0; t < T; ++t)
        for (int j = 0; j < K; ++j) {
            const int e = h_sel_[t * K + j];
            h_etok_[at[e]] = t;
            h_ew_[at[e]] = h_wts_[t * K + j];
            at[e]++;
        }
    WL_CUDA(cudaMemcpyAsync(etok_d_, h_etok_, sizeof(int32_t) * (size_t)T * K, cudaMemcpyHostToDevice, stream_));
    WL_CUDA(cudaMemcpyAsync(ew_d_, h_ew_, sizeof(float) * (size_t)T * K, cudaMemcpyHostToDevice, stream_));
    WL_CUDA(cudaMemsetAsync(moe_out_, 0, sizeof(float) * (size_t)T * E, stream_));
    for (int e = 0; e < NE; ++e) {
        const int n = count[e];
        if (n == 0) continue;
        stats_.expert_runs++;
        if (e - e_lo_ < 0 || e - e_lo_ >= e_n_) continue;     // another GPU's expert (tensor parallelism)
        const int32_t* toks = etok_d_ + start[e];
        k::gather_rows(xe_, xn_, toks, n, E, stream_);
        matmul(slice(L.gate_exps, e - e_lo_), xe_, n, ge_);
        matmul(slice(L.up_exps, e - e_lo_), xe_, n, ue_, 0, true);
        k::swiglu(ge_, ue_, (int64_t)n * X, stream_);
        matmul(slice(L.down_exps, e - e_lo_), ge_, n, ye_);
        k::scatter_add(moe_out_, ye_, toks, ew_d_ + start[e], n, E, stream_);
    }
    if (L.sh_gate.present() && tp_rank_ == 0) {     // the shared expert once (on the first GPU under TP)
        const int SF = L.sh_gate.rows;
        matmul(L.sh_gate, xn_, T, g_);
        matmul(L.sh_up, xn_, T, u_, 0, true);
        k::swiglu(g_, u_, (int64_t)T * SF, stream_);
        matmul(L.sh_down, g_, T, o_);
        if (L.sh_gate_inp.present()) matmul(L.sh_gate_inp, xn_, T, sh_gl_);
        k::shared_expert_add(moe_out_, o_, L.sh_gate_inp.present() ? sh_gl_ : nullptr, T, E, stream_);
    }
    WL_CUDA(cudaMemcpyAsync(o_, moe_out_, sizeof(float) * (size_t)T * E, cudaMemcpyDeviceToDevice, stream_));
    all_reduce(o_, (int64_t)T * E);         // the sum over the GPUs' experts (no-op on one GPU)
}

// Layer (src/Transformer.cs:177-232).
void Model::layer(int l, int T, int max_n)
{
    const LayerW& L = L_[l];
    const int E = c_.embd, QD = c_.qdim(), KD = c_.kvdim(), HD = c_.head_dim;
    const float rs = c_.residual_scale != 0.f ? c_.residual_scale : 1.f;
    const int64_t n = (int64_t)T * E;
    if (c_.post_norms) {
        WL_CUDA(cudaMemcpyAsync(xn_, x_, sizeof(float) * n, cudaMemcpyDeviceToDevice, stream_));
        prep_x_ = nullptr;
    } else {
        pre_norm(T, L.attn_norm, L.q.tiles != nullptr);
    }
    // at decode the small v matvec runs on a side stream beside the q+k launch (it reads the same prepared input and
    // writes only v), filling the SMs that the q+k launch's last CTAs leave idle; RoPE waits for both
    const bool fork = T <= 8 && L.v.tiles && !streamed_ && prep_x_ == xn_ && prep_nc_ == T && prep_cols_ == L.v.cols;
    if (fork) {
        WL_CUDA(cudaEventRecord(fork_ev_, stream_));
        WL_CUDA(cudaStreamWaitEvent(side_, fork_ev_, 0));
        std::swap(stream_, side_);
        try {
            matmul(L.v, xn_, T, v_, 0, true);
        } catch (...) {
            std::swap(stream_, side_);
            throw;
        }
        std::swap(stream_, side_);
        WL_CUDA(cudaEventRecord(join_ev_, side_));
        matmul2(L.q, L.k, xn_, T, q_, k_);
        WL_CUDA(cudaStreamWaitEvent(stream_, join_ev_, 0));
    } else {
        matmul2(L.q, L.k, xn_, T, q_, k_);
        matmul(L.v, xn_, T, v_, 0, true);
    }
    if (L.qb.present()) k::add_bias(q_, L.qb.d, T, QD, stream_);
    if (L.kb.present()) k::add_bias(k_, L.kb.d, T, KD, stream_);
    if (L.vb.present()) k::add_bias(v_, L.vb.d, T, KD, stream_);
    const int rm = profile_begin();
    bool roped = false;
    if (c_.qk_norm_full) {
        k::rmsnorm(q_, T, QD, L.q_norm.d, c_.rms_eps, q_, stream_);
        k::rmsnorm(k_, T, KD, L.k_norm.d, c_.rms_eps, k_, stream_);
    } else if (c_.qk_norm) {
        // per-head norms and the rope in one kernel where the rope covers whole NEOX heads (qwen3, qwen3moe)
        roped = k::qknorm_rope_append(q_, k_, v_, T, c_.heads, c_.kv_heads, HD, c_.rope_dims, c_.rope_neox ? 1 : 0,
                                      L.q_norm.d, L.k_norm.d, c_.rms_eps, pos_d_, rope_table_, rows_d_, l, stream_);
        if (!roped) {
            k::rmsnorm(q_, T * c_.heads, HD, L.q_norm.d, c_.rms_eps, q_, stream_);
            k::rmsnorm(k_, T * c_.kv_heads, HD, L.k_norm.d, c_.rms_eps, k_, stream_);
        }
    }
    // a one-row step leaves RoPE and the KV append to the attention kernel (same bits, one launch fewer): the row's
    // new position is read by no CTA but the one that writes it
    const bool rope_in_attention = !roped && T == 1 && !c_.qk_norm_full && c_.rope_dims >= 2 && c_.rope_dims % 2 == 0 &&
                                   c_.rope_dims <= HD;
    if (!roped && !rope_in_attention)
        k::rope_append(q_, k_, v_, T, c_.heads, c_.kv_heads, HD, c_.rope_dims, c_.rope_neox ? 1 : 0, pos_d_,
                       rope_table_, rows_d_, l, stream_);
    profile_end(rm, WL_PROFILE_ROPE, 0.0);
    const k::AttnRope ar_rope{k_, v_, rope_table_, c_.rope_dims, c_.rope_neox ? 1 : 0};
    const float scale = c_.attention_scale != 0.f ? c_.attention_scale : 1.f / (float)std::sqrt((double)HD);
    // the o matvec's activations come out of the attention combine when it can prepare them
    const bool want_prep = L.o.tiles && T <= 8 && xprep_buf_;
    k::XPrep ap{};
    if (want_prep) ap = k::xprep_view(xprep_buf_, QD, T);
    const int mark = profile_begin();
    const bool prepped = k::attention(q_, T, c_.heads, c_.kv_heads, HD, scale, rows_d_, l, pos_d_, att_part_, att_,
                                      want_prep ? &ap : nullptr, stream_, rope_in_attention ? &ar_rope : nullptr);
    profile_end(mark, WL_PROFILE_ATTENTION, 0.0);
    prep_x_ = nullptr;
    if (prepped) { prep_x_ = att_; prep_cols_ = QD; prep_nc_ = T; }
    matmul_reduce(L.o, att_, T);
    if (c_.post_norms) {
        k::rmsnorm(o_, T, E, L.post_attn_norm.d, c_.rms_eps, o_, stream_);
        k::residual(x_, o_, rs, n, stream_);
        WL_CUDA(cudaMemcpyAsync(xn_, x_, sizeof(float) * n, cudaMemcpyDeviceToDevice, stream_));
        prep_x_ = nullptr;
    } else {
        pending_residual_ = true;           // x += o happens inside the ffn norm
        pre_norm(T, L.ffn_norm, L.moe ? moe_on_device(L, T) : L.gate.tiles != nullptr);
    }
    if (L.moe) {
        if (moe_on_device(L, T)) ffn_moe_device(L, T);
        else ffn_moe(L, T);
    } else {
        ffn_dense(L, T);
    }
    if (c_.post_norms) {
        k::rmsnorm(o_, T, E, L.post_ffw_norm.d, c_.rms_eps, o_, stream_);
        k::residual(x_, o_, rs, n, stream_);
    } else {
        pending_residual_ = true;           // x += o happens inside the next norm (next layer or the head)
    }
}

// The pre-norm of a sublayer: x += o (the previous sublayer's output, when pending), xn = RmsNormRows(x) * w, and,
// for up to eight rows read by a tensor-core matvec, xn's prepared activations, all in one kernel when the row
// length allows.
void Model::pre_norm(int T, const Vec& w, bool prep_for_mma)
{
    const int E = c_.embd;
    const float rs = c_.residual_scale != 0.f ? c_.residual_scale : 1.f;
    prep_x_ = nullptr;
    const int nm = profile_begin();
    if (k::norm_prep_supported(E)) {
        const bool prep = prep_for_mma && T <= 8 && xprep_buf_;
        k::XPrep p{};
        if (prep) p = k::xprep_view(xprep_buf_, E, T);
        k::ArIn ar{};
        const bool fused = pending_residual_ && pending_ar_in(T, 0, &ar);
        const bool moe = pending_residual_ && pending_moe_;
        k::norm_prep(x_, pending_residual_ ? o_ : nullptr, rs, T, E, w.d, c_.rms_eps, xn_, prep ? &p : nullptr, stream_,
                     fused ? &ar : nullptr, moe ? &moe_in_ : nullptr);
        if (prep) { prep_x_ = xn_; prep_cols_ = E; prep_nc_ = T; }
    } else {
        if (pending_residual_) k::residual(x_, o_, rs, (int64_t)T * E, stream_);
        k::rmsnorm(x_, T, E, w.d, c_.rms_eps, xn_, stream_);
    }
    profile_end(nm, WL_PROFILE_NORM, 0.0);
    pending_residual_ = false;
    pending_moe_ = false;
}

// Head (src/Transformer.cs:112-125): final norm and output matrix for rows first..T-1.
void Model::head(int T, int first)
{
    const int E = c_.embd, n = T - first;
    const float rs = c_.residual_scale != 0.f ? c_.residual_scale : 1.f;
    prep_x_ = nullptr;
    if (k::norm_prep_supported(E)) {
        const bool prep = output_.tiles && n <= 8 && xprep_buf_;
        k::XPrep p{};
        if (prep) p = k::xprep_view(xprep_buf_, E, n);
        k::ArIn ar{};
        const bool fused = pending_residual_ && pending_ar_in(n, first, &ar);
        k::MoeIn mi = moe_in_;          // the head's rows first.. take their own pairs
        mi.y += (int64_t)first * mi.K * E;
        mi.sel += (int64_t)first * mi.K;
        mi.wts += (int64_t)first * mi.K;
        const bool moe = pending_residual_ && pending_moe_;
        k::norm_prep(x_ + (int64_t)first * E, pending_residual_ ? o_ + (int64_t)first * E : nullptr, rs, n, E,
                     out_norm_.d, c_.rms_eps, xn_, prep ? &p : nullptr, stream_, fused ? &ar : nullptr,
                     moe ? &mi : nullptr);
        if (prep) { prep_x_ = xn_; prep_cols_ = E; prep_nc_ = n; }
    } else {
        if (pending_residual_) k::residual(x_, o_, rs, (int64_t)T * E, stream_);
        k::rmsnorm(x_ + (int64_t)first * E, n, E, out_norm_.d, c_.rms_eps, xn_, stream_);
    }
    pending_residual_ = false;
    pending_moe_ = false;
    if (comm_) {
        // this rank's vocabulary rows, then every rank's gathered and laid out as [n][vocab]
        matmul(output_, xn_, n, logits_part_, 0, true, vocab_part_);
        const int mark = profile_begin();
        comm_->allgather(logits_part_, logits_all_, (int64_t)n * vocab_part_ * 4, stream_);
        profile_end(mark, WL_PROFILE_ALLREDUCE, 4.0 * n * vocab_part_ * (tp_size_ - 1));
        k::vocab_gather(logits_all_, tp_size_, n, vocab_part_, c_.vocab, logits_, stream_);
    } else {
        matmul(output_, xn_, n, logits_, 0, true);
    }
    if (c_.logit_scale != 0.f) k::scale(logits_, 1.f / c_.logit_scale, (int64_t)n * c_.vocab, stream_);
}

// Token ids, positions and KV-cache rows of one step to the device (pinned staging, async on the model's stream).
void Model::upload_step(int T, const RowKV* rows, const int32_t* pos, const int32_t* tokens)
{
    for (int t = 0; t < T; ++t) {
        h_tok_[t] = tokens[t];
        h_pos_[t] = pos[t];
        h_rows_[t] = rows[t];
    }
    WL_CUDA(cudaMemcpyAsync(tok_d_, h_tok_, sizeof(int32_t) * T, cudaMemcpyHostToDevice, stream_));
    WL_CUDA(cudaMemcpyAsync(pos_d_, h_pos_, sizeof(int32_t) * T, cudaMemcpyHostToDevice, stream_));
    WL_CUDA(cudaMemcpyAsync(rows_d_, h_rows_, sizeof(RowKV) * T, cudaMemcpyHostToDevice, stream_));
}

// Embedding, every layer and the head, all on the device (no cancel or progress points).
void Model::step_device(int T, int first, int max_n)
{
    begin_step(T);
    for (int l = 0; l < c_.layers; ++l) {
        stage_acquire(l);
        layer(l, T, max_n);
        stage_release(l);
    }
    stage_acquire(c_.layers);
    head(T, first);
    stage_release(c_.layers);
}

int32_t Model::run(int T, const std::vector<RowKV>& rows, const std::vector<int32_t>& pos, const int32_t* tokens,
                   int first, float* out, int32_t* ids, volatile const int32_t* cancel, wl_progress_fn progress,
                   void* user)
{
    const auto t0 = std::chrono::steady_clock::now();
    for (int t = 0; t < T; ++t)
        if (tokens[t] < 0 || tokens[t] >= c_.vocab)
            WL_THROW(WL_EINVAL, "Token id " + std::to_string(tokens[t]) + " is outside the vocabulary.");
    ensure_workspace(T, T - first);
    upload_step(T, rows.data(), pos.data(), tokens);
    int max_n = 0;
    for (int t = 0; t < T; ++t) max_n = std::max(max_n, pos[t] + 1);
    const int total = c_.layers + 1;
    const bool stop0 = stop_requested(cancel);
    if (!progress && !stop0 && graph_step(T, first)) {
        // the whole step ran as one graph; a cancel flag set meanwhile is seen by the next call
    } else if (!cancel && !progress) step_device(T, first, max_n);
    else {
        begin_step(T);
        for (int l = 0; l < c_.layers; ++l) {
            if (l == 0 ? stop0 : stop_requested(cancel)) { WL_CUDA(cudaStreamSynchronize(stream_)); return WL_CANCELLED; }
            stage_acquire(l);
            layer(l, T, max_n);
            stage_release(l);
            if (progress) { WL_CUDA(cudaStreamSynchronize(stream_)); progress(l + 1, total, user); }
        }
        if (stop_requested(cancel)) { WL_CUDA(cudaStreamSynchronize(stream_)); return WL_CANCELLED; }
        stage_acquire(c_.layers);
        head(T, first);
        stage_release(c_.layers);
    }
    if (ids && sampling_) {
        if (!sample_ws_) {
            sample_ws_ = dalloc<uint8_t>((int64_t)k::sample_workspace_bytes(c_.vocab));
            k::sample_workspace_init(sample_ws_, stream_);
        }
        for (int r = 0; r < T - first; ++r)
            k::sample(logits_ + (int64_t)r * c_.vocab, c_.vocab, sampling_->temperature[r], sampling_->top_p[r],
                      sampling_->draw[r], sample_ws_, ids_d_ + r, stream_);
        WL_CUDA(cudaMemcpyAsync(h_ids_, ids_d_, sizeof(int32_t) * (size_t)(T - first), cudaMemcpyDeviceToHost, stream_));
        WL_CUDA(cudaStreamSynchronize(stream_));
        for (int r = 0; r < T - first; ++r) ids[r] = h_ids_[r];
    } else if (ids) {
        k::argmax(logits_, c_.vocab, T - first, amax_key_, amax_count_, ids_d_, nullptr, nullptr, stream_);
        WL_CUDA(cudaMemcpyAsync(h_ids_, ids_d_, sizeof(int32_t) * (size_t)(T - first), cudaMemcpyDeviceToHost, stream_));
        WL_CUDA(cudaStreamSynchronize(stream_));
        for (int r = 0; r < T - first; ++r) ids[r] = h_ids_[r];
    } else {
        WL_CUDA(cudaMemcpyAsync(out, logits_, sizeof(float) * (size_t)(T - first) * c_.vocab, cudaMemcpyDeviceToHost, stream_));
        WL_CUDA(cudaStreamSynchronize(stream_));
    }
    check_device_error();
    flush_profile();
    if (progress) progress(total, total, user);
    stats_.tokens += T;
    stats_.last_forward_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return WL_OK;
}

// ---------------------------------------------------------------------------------------------------------------------
// CUDA graphs: a decode step of T <= 8 rows is captured once per (T, first logit row) and replayed. The graph reads
// token ids, positions and KV-cache rows from the fixed device buffers upload_step fills, and sizes attention for the
// whole context, so one graph serves every step of that shape until the workspaces are reallocated. MoE layers
// (host-side expert grouping), profiling and per-layer progress callbacks run eagerly.
// ---------------------------------------------------------------------------------------------------------------------
bool Model::graphable(int T) const
{
    if (!use_graphs_ || profiling_ || streamed_ || T > 8) return false;
    for (const LayerW& L : L_)
        if (L.moe && !moe_on_device(L, T)) return false;   // the host-side expert grouping syncs
    return true;
}

// True when a graph for (T, first) exists or could be captured now (after one eager run of that shape).
bool Model::graph_ready(int T, int first)
{
    if (!graphable(T)) return false;
    for (const GraphEntry& g : graphs_)
        if (g.T == T && g.first == first && g.gen == ws_gen_) return true;
    // capture: kernels set their launch attributes during an eager run first; that run repeats the step the graph
    // then runs, so the experts it counts are taken back
    if (expert_count_d_)
        WL_CUDA(cudaMemcpyAsync(expert_count_d_ + 1, expert_count_d_, sizeof(unsigned long long),
                                cudaMemcpyDeviceToDevice, stream_));
    step_device(T, first, max_context_);
    if (expert_count_d_)
        WL_CUDA(cudaMemcpyAsync(expert_count_d_, expert_count_d_ + 1, sizeof(unsigned long long),
                                cudaMemcpyDeviceToDevice, stream_));
    const int64_t l0 = k::launches();
    cudaGraph_t graph = nullptr;
    WL_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    try {
        step_device(T, first, max_context_);
    } catch (...) {
        cudaStreamEndCapture(stream_, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
    }
    WL_CUDA(cudaStreamEndCapture(stream_, &graph));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    WL_CUDA(e);
    const int64_t nodes = k::launches() - l0;
    k::uncount_launches(nodes);      // captured, not run: replays count them
    graphs_.push_back(GraphEntry{T, first, ws_gen_, exec, nodes});
    return true;
}

bool Model::graph_step(int T, int first)
{
    if (!graph_ready(T, first)) return false;
    for (const GraphEntry& g : graphs_)
        if (g.T == T && g.first == first && g.gen == ws_gen_) {
            WL_CUDA(cudaGraphLaunch(g.exec, stream_));
            graph_launches_ += g.nodes;
            return true;
        }
    return false;
}

void Model::drop_graphs()
{
    for (GraphEntry& g : graphs_) cudaGraphExecDestroy(g.exec);
    graphs_.clear();
}

double Model::bench_decode(Seq* const* seqs, int N, int steps)
{
    if (N <= 0 || steps <= 0) WL_THROW(WL_EINVAL, "wl_bench_decode: N and steps must be positive");
    WL_CUDA(cudaSetDevice(device_));
    std::vector<int32_t> len(N);
    int max_len = 0;
    for (int i = 0; i < N; ++i) {
        if (!seqs[i] || seqs[i]->model != this) WL_THROW(WL_EINVAL, "wl_bench_decode: a sequence of another model");
        len[i] = seqs[i]->length;
        if (len[i] + steps > max_context_) WL_THROW(WL_EINVAL, "wl_bench_decode: the steps do not fit the context");
        reserve(seqs[i], len[i] + steps);
        max_len = std::max(max_len, len[i]);
    }
    ensure_workspace(N, N);
    // every step's positions up front, so the timed loop copies nothing from the host
    std::vector<int32_t> pos_all((size_t)steps * N), toks(N);
    std::vector<RowKV> rows(N);
    for (int i = 0; i < N; ++i) {
        const int64_t stride = (int64_t)seqs[i]->capacity * c_.kvdim();
        rows[i] = RowKV{seqs[i]->kv, seqs[i]->kv + (int64_t)c_.layers * stride, stride};
        toks[i] = (int32_t)((1103515245u * (uint32_t)(i + 1) + 12345u) % (uint32_t)c_.vocab);
        for (int s = 0; s < steps; ++s) pos_all[(size_t)s * N + i] = len[i] + s;
    }
    int32_t* pos_all_d = dalloc<int32_t>((int64_t)steps * N);
    WL_CUDA(cudaMemcpy(pos_all_d, pos_all.data(), pos_all.size() * 4, cudaMemcpyHostToDevice));
    upload_step(N, rows.data(), pos_all.data(), toks.data());
    // ForwardBatch steps (every row as if alone); a graph is captured (or found) before the timed loop so capture
    // costs are not timed
    struct EachToken {
        bool& f;
        explicit EachToken(bool& b) : f(b) { f = true; }
        ~EachToken() { f = false; }
    } each(each_token_);
    const bool graphs = graph_ready(N, 0);
    cudaEvent_t e0, e1;
    WL_CUDA(cudaEventCreate(&e0));
    WL_CUDA(cudaEventCreate(&e1));
    WL_CUDA(cudaEventRecord(e0, stream_));
    for (int s = 0; s < steps; ++s) {
        WL_CUDA(cudaMemcpyAsync(pos_d_, pos_all_d + (size_t)s * N, sizeof(int32_t) * N, cudaMemcpyDeviceToDevice, stream_));
        if (!graphs || !graph_step(N, 0)) step_device(N, 0, max_len + s + 1);
    }
    WL_CUDA(cudaEventRecord(e1, stream_));
    WL_CUDA(cudaEventSynchronize(e1));
    float ms = 0.f;
    WL_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(pos_all_d);
    check_device_error();
    flush_profile();
    for (int i = 0; i < N; ++i) seqs[i]->length = len[i] + steps;
    stats_.tokens += (int64_t)N * steps;
    return ms;
}

// The Q4_K matvec launches of one decode step of T rows, with the step's weights, shapes, column counts, pairings and
// order (q and k, o, gate and up, down per layer), captured into a CUDA graph and replayed `steps` times alone: the
// dominant kernel's own rate, with the programmatic-launch overlap between consecutive matvecs that the step has
// between its kernels. The activations are whatever the prepared-activation buffer holds (the timing does not depend
// on them); outputs go to the model's scratch rows. Returns the device milliseconds of the replays and, through bytes,
// the matvecs' algorithmic bytes per step (weights + activations in + outputs).
double Model::bench_matvecs(int T, int steps, double* bytes)
{
    if (T < 1 || T > 8 || steps <= 0) WL_THROW(WL_EINVAL, "wl_bench_matvecs: 1 <= T <= 8 and steps > 0");
    WL_CUDA(cudaSetDevice(device_));
    ensure_workspace(T, T);
    if (!xprep_buf_) WL_THROW(WL_EUNSUPPORTED, "wl_bench_matvecs: the model has no tensor-core matvec");
    double total = 0.0;
    auto q4 = [](const Weight& w) { return w.present() && w.type == 12 && w.tiles; };
    auto count = [&](const Weight& w) {
        if (q4(w)) total += (double)w.rows * w.row_bytes + 4.0 * T * ((double)w.cols + w.rows);
    };
    // the launches of one step; the prepared activations are taken as already made for every input, so no prep
    // kernel runs (matmul and matmul2 reuse a matching prepared input)
    auto launches = [&]() {
        for (const LayerW& L : L_) {
            if (L.moe) continue;
            float* dummy = xn_;
            auto ready = [&](int cols) { prep_x_ = dummy; prep_cols_ = cols; prep_nc_ = T; };
            if (q4(L.q) && q4(L.k)) { ready(L.q.cols); matmul2(L.q, L.k, dummy, T, q_, k_); }
            if (q4(L.o)) { ready(L.o.cols); matmul(L.o, dummy, T, o_, 0, true); }
            if (q4(L.gate) && q4(L.up)) { ready(L.gate.cols); matmul2(L.gate, L.up, dummy, T, g_, u_); }
            if (q4(L.down)) { ready(L.down.cols); matmul(L.down, dummy, T, o_, 0, true); }
        }
        prep_x_ = nullptr;
    };
    for (const LayerW& L : L_) {
        if (L.moe) continue;
        if (q4(L.q) && q4(L.k)) { count(L.q); count(L.k); }
        count(L.o);
        if (q4(L.gate) && q4(L.up)) { count(L.gate); count(L.up); }
        count(L.down);
    }
    launches();                         // eager first: kernel attributes are set outside the capture
    const int64_t l0 = k::launches();
    cudaGraph_t graph = nullptr;
    WL_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    try {
        launches();
    } catch (...) {
        cudaStreamEndCapture(stream_, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
    }
    WL_CUDA(cudaStreamEndCapture(stream_, &graph));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    WL_CUDA(e);
    const int64_t nodes = k::launches() - l0;
    k::uncount_launches(nodes);
    WL_CUDA(cudaGraphLaunch(exec, stream_));        // warm
    cudaEvent_t e0, e1;
    WL_CUDA(cudaEventCreate(&e0));
    WL_CUDA(cudaEventCreate(&e1));
    WL_CUDA(cudaEventRecord(e0, stream_));
    for (int i = 0; i < steps; ++i) WL_CUDA(cudaGraphLaunch(exec, stream_));
    WL_CUDA(cudaEventRecord(e1, stream_));
    WL_CUDA(cudaEventSynchronize(e1));
    float ms = 0.f;
    WL_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(exec);
    graph_launches_ += nodes * (steps + 1);
    check_device_error();
    if (bytes) *bytes = total;
    return ms;
}

// ---------------------------------------------------------------------------------------------------------------------
// profiling: CUDA events around every matvec/matmul launch on the model's stream
// ---------------------------------------------------------------------------------------------------------------------
void Model::set_profiling(bool on)
{
    WL_CUDA(cudaSetDevice(device_));
    WL_CUDA(cudaStreamSynchronize(stream_));
    flush_profile();
    profiling_ = on;
    if (on) for (auto& p : prof_) p = wl_profile_entry{};
}

void Model::flush_profile()
{
    if (marks_.empty()) return;
    WL_CUDA(cudaStreamSynchronize(stream_));
    for (const ProfileMark& m : marks_) {
        float ms = 0.f;
        WL_CUDA(cudaEventElapsedTime(&ms, m.start, m.stop));
        wl_profile_entry& e = prof_[m.type & 63];
        e.launches++;
        e.ms += ms;
        e.bytes += m.bytes;
        event_pool_.push_back(m.start);
        event_pool_.push_back(m.stop);
    }
    marks_.clear();
}

wl_profile_entry Model::profile(int type)
{
    flush_profile();
    return prof_[type & 63];
}

// Transformer.Forward (src/Transformer.cs:83-109).
int32_t Model::forward(Seq* sq, const int32_t* tokens, int T, int pos0, bool all_logits, float* out,
                       volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    return forward_impl(sq, tokens, T, pos0, all_logits, out, nullptr, cancel, progress, user);
}

int32_t Model::forward_argmax(Seq* sq, const int32_t* tokens, int T, int pos0, bool all_rows, int32_t* ids,
                              volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    return forward_impl(sq, tokens, T, pos0, all_rows, nullptr, ids, cancel, progress, user);
}

namespace {
// Sets a model's sampling options for one call and clears them however the call ends.
struct SamplingScope {
    const Model::SampleRows*& slot;
    SamplingScope(const Model::SampleRows*& s, const Model::SampleRows* v) : slot(s) { slot = v; }
    ~SamplingScope() { slot = nullptr; }
};

void check_sample_rows(const Model::SampleRows& sr, int n)
{
    if (!sr.temperature || !sr.top_p || !sr.draw) WL_THROW(WL_EINVAL, "Sampling needs a temperature, top_p and draw for each row.");
    for (int r = 0; r < n; ++r)
        if (sr.temperature[r] > 0.0 && !(sr.draw[r] >= 0.0 && sr.draw[r] < 1.0))
            WL_THROW(WL_EINVAL, "A sampling draw must be in [0, 1).");
}
}  // namespace

int32_t Model::forward_sample(Seq* sq, const int32_t* tokens, int T, int pos0, const SampleRows& sr, int32_t* id,
                              volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    check_sample_rows(sr, 1);
    SamplingScope scope(sampling_, &sr);
    return forward_impl(sq, tokens, T, pos0, false, nullptr, id, cancel, progress, user);
}

int32_t Model::forward_batch_sample(Seq* const* seqs, const int32_t* tokens, int N, const SampleRows& sr, int32_t* ids,
                                    volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    check_sample_rows(sr, N);
    SamplingScope scope(sampling_, &sr);
    return forward_batch_impl(seqs, tokens, N, nullptr, ids, cancel, progress, user);
}

int32_t Model::forward_impl(Seq* sq, const int32_t* tokens, int T, int pos0, bool all_logits, float* out, int32_t* ids,
                            volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    if (!sq) sq = own_;
    if (T <= 0) WL_THROW(WL_EINVAL, "No tokens to run.");
    if (pos0 < 0 || pos0 > sq->length) WL_THROW(WL_EINVAL, "pos0 is past the cached positions.");
    if (pos0 + T > max_context_)
        WL_THROW(WL_EINVAL, "The prompt and reply need " + std::to_string(pos0 + T) + " positions; the context is " + std::to_string(max_context_) + ".");
    WL_CUDA(cudaSetDevice(device_));
    sq->length = pos0;
    reserve(sq, pos0 + T);
    const int64_t stride = (int64_t)sq->capacity * c_.kvdim();
    std::vector<RowKV> rows(T, RowKV{sq->kv, sq->kv + (int64_t)c_.layers * stride, stride});
    std::vector<int32_t> pos(T);
    for (int t = 0; t < T; ++t) pos[t] = pos0 + t;
    stats_.forward_calls++;
    const int32_t st = run(T, rows, pos, tokens, all_logits ? 0 : T - 1, out, ids, cancel, progress, user);
    if (st == WL_OK) sq->length = pos0 + T;
    return st;
}

// Transformer.ForwardBatch (src/Transformer.cs:132-170).
int32_t Model::forward_batch(Seq* const* seqs, const int32_t* tokens, int N, float* out, volatile const int32_t* cancel,
                             wl_progress_fn progress, void* user)
{
    return forward_batch_impl(seqs, tokens, N, out, nullptr, cancel, progress, user);
}

int32_t Model::forward_batch_argmax(Seq* const* seqs, const int32_t* tokens, int N, int32_t* ids,
                                    volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    return forward_batch_impl(seqs, tokens, N, nullptr, ids, cancel, progress, user);
}

int32_t Model::forward_batch_impl(Seq* const* seqs, const int32_t* tokens, int N, float* out, int32_t* ids,
                                  volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    if (N <= 0 || !seqs) WL_THROW(WL_EINVAL, "ForwardBatch needs one token for each sequence.");
    if (N > max_batch_) WL_THROW(WL_EINVAL, "ForwardBatch takes at most " + std::to_string(max_batch_) + " sequences.");
    WL_CUDA(cudaSetDevice(device_));
    std::vector<int32_t> pos(N);
    for (int i = 0; i < N; ++i) {
        Seq* sq = seqs[i];
        if (!sq || sq->model != this) WL_THROW(WL_EINVAL, "A sequence of another model was passed.");
        for (int j = 0; j < i; ++j) if (seqs[j] == sq) WL_THROW(WL_EINVAL, "A sequence can take one token per batch step.");
        if (sq->length + 1 > max_context_)
            WL_THROW(WL_EINVAL, "The prompt and reply need " + std::to_string(sq->length + 1) + " positions; the context is " + std::to_string(max_context_) + ".");
        pos[i] = sq->length;
    }
    std::vector<RowKV> rows(N);
    for (int i = 0; i < N; ++i) {
        reserve(seqs[i], pos[i] + 1);
        const int64_t stride = (int64_t)seqs[i]->capacity * c_.kvdim();
        rows[i] = RowKV{seqs[i]->kv, seqs[i]->kv + (int64_t)c_.layers * stride, stride};
    }
    stats_.batch_calls++;
    // MatMulEach (src/Transformer.cs:544-561): each row bit-identical to running alone, so no GEMM for this step
    each_token_ = true;
    int32_t st;
    try {
        st = run(N, rows, pos, tokens, 0, out, ids, cancel, progress, user);
    } catch (...) {
        each_token_ = false;
        throw;
    }
    each_token_ = false;
    if (st == WL_OK) for (int i = 0; i < N; ++i) seqs[i]->length = pos[i] + 1;
    return st;
}

// Several sequences' new tokens in one pass. Every row carries its own position and KV-cache row table, and within a
// layer all rows' K/V are appended before any row attends, so the order of the rows is free: the rows before each
// sequence's last token come first, then the N last rows in sequence order, and the head runs on those N only.
int32_t Model::forward_mixed(Seq* const* seqs, const int32_t* counts, int N, const int32_t* tokens, float* out,
                             int32_t* ids, volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    if (N <= 0 || !seqs || !counts) WL_THROW(WL_EINVAL, "A mixed step needs at least one sequence.");
    if (N > max_batch_) WL_THROW(WL_EINVAL, "A mixed step takes at most " + std::to_string(max_batch_) + " sequences.");
    WL_CUDA(cudaSetDevice(device_));
    int64_t total = 0;
    for (int i = 0; i < N; ++i) {
        Seq* sq = seqs[i];
        if (!sq || sq->model != this) WL_THROW(WL_EINVAL, "A sequence of another model was passed.");
        for (int j = 0; j < i; ++j) if (seqs[j] == sq) WL_THROW(WL_EINVAL, "A sequence can appear once in a mixed step.");
        if (counts[i] <= 0) WL_THROW(WL_EINVAL, "Every sequence of a mixed step needs at least one token.");
        if ((int64_t)sq->length + counts[i] > max_context_)
            WL_THROW(WL_EINVAL, "The prompt and reply need " + std::to_string((int64_t)sq->length + counts[i]) +
                                    " positions; the context is " + std::to_string(max_context_) + ".");
        total += counts[i];
    }
    if (total > (1 << 20)) WL_THROW(WL_EINVAL, "A mixed step of more than 2^20 tokens.");
    const int T = (int)total;
    std::vector<RowKV> row(N);
    for (int i = 0; i < N; ++i) {
        reserve(seqs[i], seqs[i]->length + counts[i]);
        const int64_t stride = (int64_t)seqs[i]->capacity * c_.kvdim();
        row[i] = RowKV{seqs[i]->kv, seqs[i]->kv + (int64_t)c_.layers * stride, stride};
    }
    std::vector<RowKV> rows((size_t)T);
    std::vector<int32_t> pos((size_t)T), toks((size_t)T);
    int k = 0;
    int64_t off = 0;
    for (int i = 0; i < N; ++i) {
        for (int j = 0; j + 1 < counts[i]; ++j, ++k) {
            rows[k] = row[i];
            pos[k] = seqs[i]->length + j;
            toks[k] = tokens[off + j];
        }
        off += counts[i];
    }
    off = 0;
    for (int i = 0; i < N; ++i, ++k) {
        off += counts[i];
        rows[k] = row[i];
        pos[k] = seqs[i]->length + counts[i] - 1;
        toks[k] = tokens[off - 1];
    }
    stats_.batch_calls++;
    const int32_t st = run(T, rows, pos, toks.data(), T - N, out, ids, cancel, progress, user);
    if (st == WL_OK) for (int i = 0; i < N; ++i) seqs[i]->length += counts[i];
    return st;
}

// LayeredBackend.Generate's decode loop at temperature 0 (src/Engine.cs:187-203) with the token chained on the device:
// each step is the T = 1 pass (a CUDA graph when the model allows one) followed by the argmax, which writes the id
// to the step's slot, to the token buffer the next step embeds from, and advances the position buffer. The host
// launches `chunk` steps without waiting, then reads their ids: a stop id ends the call there (the steps launched
// after it are dropped; what they wrote to the KV cache lies past the sequence's length). The cancel flag is read
// before each chunk (under tensor parallelism by every rank, so all stop together).
int32_t Model::generate_greedy(Seq* sq, int32_t token, int max_new, const int32_t* stop, int n_stop, int chunk,
                               int32_t* ids, int32_t* n_out, volatile const int32_t* cancel)
{
    constexpr int MAX_CHUNK = 64;
    if (!sq) sq = own_;
    *n_out = 0;
    if (max_new < 0) WL_THROW(WL_EINVAL, "max_new must not be negative.");
    if (n_stop < 0 || (n_stop > 0 && !stop)) WL_THROW(WL_EINVAL, "The stop ids are missing.");
    if (chunk < 0 || chunk > MAX_CHUNK) WL_THROW(WL_EINVAL, "chunk must be 0 (the default, 16) up to 64.");
    if (token < 0 || token >= c_.vocab)
        WL_THROW(WL_EINVAL, "Token id " + std::to_string(token) + " is outside the vocabulary.");
    if (max_new == 0) return WL_OK;
    if (chunk == 0) chunk = 16;
    const int len = sq->length;
    if ((int64_t)len + max_new > max_context_)
        WL_THROW(WL_EINVAL, "The prompt and reply need " + std::to_string((int64_t)len + max_new) +
                                " positions; the context is " + std::to_string(max_context_) + ".");
    WL_CUDA(cudaSetDevice(device_));
    const auto t0 = std::chrono::steady_clock::now();
    reserve(sq, len + max_new);
    ensure_workspace(1, 1);
    if (!gen_d_) {
        gen_d_ = dalloc<int32_t>(MAX_CHUNK);
        h_gen_ = halloc<int32_t>(MAX_CHUNK);
    }
    const int64_t stride = (int64_t)sq->capacity * c_.kvdim();
    const RowKV row{sq->kv, sq->kv + (int64_t)c_.layers * stride, stride};
    upload_step(1, &row, &len, &token);
    stats_.forward_calls++;
    int done = 0;
    while (done < max_new) {
        if (stop_requested(cancel)) {
            WL_CUDA(cudaStreamSynchronize(stream_));
            sq->length = len + done;
            *n_out = done;
            return WL_CANCELLED;
        }
        const int c = std::min(chunk, max_new - done);
        for (int j = 0; j < c; ++j) {
            if (!graph_step(1, 0)) step_device(1, 0, len + done + j + 1);
            k::argmax(logits_, c_.vocab, 1, amax_key_, amax_count_, gen_d_ + j, tok_d_, pos_d_, stream_);
        }
        WL_CUDA(cudaMemcpyAsync(h_gen_, gen_d_, sizeof(int32_t) * (size_t)c, cudaMemcpyDeviceToHost, stream_));
        WL_CUDA(cudaStreamSynchronize(stream_));
        check_device_error();
        for (int j = 0; j < c; ++j) {
            ids[done] = h_gen_[j];
            ++done;
            for (int i = 0; i < n_stop; ++i)
                if (stop[i] == h_gen_[j]) {
                    sq->length = len + done;
                    *n_out = done;
                    stats_.tokens += done;
                    flush_profile();
                    return WL_OK;
                }
        }
    }
    sq->length = len + done;
    *n_out = done;
    stats_.tokens += done;
    flush_profile();
    stats_.last_forward_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return WL_OK;
}

}  // namespace wl
