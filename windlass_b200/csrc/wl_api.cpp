// The C ABI of libwindlass_cuda (include/windlass.h): argument checks, exception-to-status translation, and the
// kernel-level test exports. No function aborts or exits; failures return a status and set wl_last_error().
#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>
#include "../../include/windlass.h"
#include "wl_common.h"
#include "wl_kernels.h"
#include "wl_group.h"
#include "wl_model.h"

namespace wl { const char* last_error_cstr(); }

// m: the model, or shard 0 of g (one model spanning several GPUs in this process, wl_options.tp_rank = -1).
struct wl_model {
    wl::Model* m;
    wl::Group* g;
};
// s: the sequence, or shard 0's of a group model, shards[i] shard i's.
struct wl_seq {
    wl::Seq* s;
    wl_model* owner;
    std::vector<wl::Seq*> shards;
};

namespace {
bool in_process_group(const wl_options& o)
{
    return o.size >= (int32_t)sizeof(wl_options) && o.tp_size > 1 && o.tp_rank == -1;
}

// The sequence of shard g (shard 0: the sequence itself).
wl::Seq* shard_seq(wl_seq* seq, int g) { return g == 0 ? seq->s : seq->shards[(size_t)g]; }

void noop_progress(int32_t, int32_t, void*) {}

template <typename F> int32_t guarded(F&& f)
{
    try {
        wl::clear_error();
        return f();
    } catch (const wl::Error& e) {
        return wl::fail(e.status, e.msg);
    } catch (const std::bad_alloc&) {
        return wl::fail(WL_ENOMEM, "out of host memory");
    } catch (const std::exception& e) {
        return wl::fail(WL_EINVAL, e.what());
    } catch (...) {
        return wl::fail(WL_EINVAL, "unknown failure");
    }
}

wl_options defaults()
{
    wl_options o;
    wl_options_init(&o);
    return o;
}

// Per-device scratch of the kernel-level exports (the model keeps its own workspaces).
// Per device: the kernel-level exports' scratch, whose first word is the error word of their bounded waits, and the
// codes collected from it before it moved (it is reallocated when a call needs more).
std::mutex g_scratch_mu;
void* g_scratch[64] = {};
size_t g_scratch_size[64] = {};
int g_scratch_code[64] = {};

void* export_scratch(size_t bytes)
{
    int dev = 0;
    WL_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (dev >= 64) WL_THROW(WL_EINVAL, "device ordinal out of range");
    if (g_scratch_size[dev] < bytes) {
        if (g_scratch[dev]) {
            WL_CUDA(cudaDeviceSynchronize());
            int e = 0;
            WL_CUDA(cudaMemcpy(&e, g_scratch[dev], sizeof e, cudaMemcpyDeviceToHost));
            if (e && !g_scratch_code[dev]) g_scratch_code[dev] = e;
            cudaFree(g_scratch[dev]);
            g_scratch[dev] = nullptr;
            g_scratch_size[dev] = 0;
        }
        WL_CUDA(cudaMalloc(&g_scratch[dev], bytes));
        WL_CUDA(cudaMemset(g_scratch[dev], 0, 256));
        g_scratch_size[dev] = bytes;
    }
    return g_scratch[dev];
}

// The forward pass's matvec rule: the tensor-core kernel where the format allows (the weights repacked into tiles,
// 8 columns per launch, activations prepared once per chunk), else the CUDA-core kernel. force_cuda_cores selects
// the latter.
void run_matvec(int type, const uint8_t* w, int rows, int cols, const float* x, int ncols, float* y, bool force_cuda_cores,
                cudaStream_t s, bool allow_gemm = true)
{
    const int64_t rb = wl::row_bytes_of(type, cols);
    if (!force_cuda_cores && allow_gemm && ncols >= wl::k::gemm_min_rows(type) && wl::k::gemm_supported(type, cols)) {
        // scratch: [error word | the activations' bf16 planes | the weights repacked into tiles]
        const size_t xb = (wl::k::gemm_scratch_bytes(ncols, cols) + 255) / 256 * 256;
        uint8_t* scratch = (uint8_t*)export_scratch(256 + xb + (size_t)wl::k::tile_bytes(type, rows, cols));
        int* err = (int*)scratch;
        uint8_t* tiles = scratch + 256 + xb;
        // the tiles are written by a kernel here, and the GEMM reads weights before its grid-dependency wait: the
        // memset between them (not a kernel) makes the GEMM start only once the repack has completed
        wl::k::make_tiles(type, w, rows, cols, rb, tiles, s);
        WL_CUDA(cudaMemsetAsync(scratch + 128, 0, sizeof(int), s));   // orders the launches behind all earlier work
        wl::k::gemm_tiles(type, tiles, 0, rows, cols, x, cols, ncols, y, rows, scratch + 256, err, s);
        return;
    }
    if (!force_cuda_cores && wl::k::tiles_supported(type, cols) && (uintptr_t)x % 16 == 0) {
        // scratch: [error word | prepared activations | the weights repacked into tiles]
        const size_t xb = (wl::k::xprep_bytes(cols, 8) + 255) / 256 * 256;
        uint8_t* scratch = (uint8_t*)export_scratch(256 + xb + (size_t)wl::k::tile_bytes(type, rows, cols));
        int* err = (int*)scratch;
        uint8_t* tiles = scratch + 256 + xb;
        // as above: the memset after the repack keeps the matvecs' early weight reads behind it
        wl::k::make_tiles(type, w, rows, cols, rb, tiles, s);
        WL_CUDA(cudaMemsetAsync(scratch + 128, 0, sizeof(int), s));   // orders the launches behind all earlier work
        for (int c0 = 0; c0 < ncols; c0 += 8) {
            const int nc = ncols - c0 < 8 ? ncols - c0 : 8;
            const wl::k::XPrep p = wl::k::xprep_view(scratch + 256, cols, nc);
            wl::k::xprep(x + (int64_t)c0 * cols, cols, cols, nc, p, s);
            wl::k::matvec_tiles(type, tiles, 0, rows, cols, p, y + (int64_t)c0 * rows, rows, err, s);
        }
        return;
    }
    wl::k::matvec(type, w, rb, rows, cols, x, cols, ncols, y, rows, s);
}
}  // namespace

extern "C" {

void wl_options_init(wl_options* opt)
{
    if (!opt) return;
    memset(opt, 0, sizeof *opt);
    opt->size = (int32_t)sizeof(wl_options);
    opt->device = 0;
    opt->max_context = 0;
    opt->max_batch = 64;
    opt->resident = -1;
    opt->prefill_path = 0;
    opt->use_graphs = 1;
    opt->tp_size = 1;
    opt->tp_rank = 0;
}

const char* wl_last_error(void) { return wl::last_error_cstr(); }
const char* wl_version(void) { return "windlass-cuda 0.1 (sm_100a)"; }

int32_t wl_tp_unique_id(uint8_t* id, int32_t bytes)
{
    return guarded([&]() -> int32_t {
        if (!id || bytes < wl::TP_ID_BYTES) return wl::fail(WL_EINVAL, "wl_tp_unique_id: id needs 128 bytes");
        wl::Comm::unique_id(id);
        return WL_OK;
    });
}

int32_t wl_open(const char* path, const wl_options* opt, wl_model** out)
{
    return guarded([&]() -> int32_t {
        if (!path || !out) return wl::fail(WL_EINVAL, "wl_open: path and out are required");
        *out = nullptr;
        const wl_options o = opt ? *opt : defaults();
        if (in_process_group(o)) {
            wl::Group* g = wl::Group::open(path, nullptr, o);
            *out = new wl_model{&g->shard(0), g};
            return WL_OK;
        }
        wl::Model* m = wl::Model::open_file(path, o);
        *out = new wl_model{m, nullptr};
        return WL_OK;
    });
}

int32_t wl_open_synthetic(const wl_synth_spec* spec, const wl_options* opt, wl_model** out)
{
    return guarded([&]() -> int32_t {
        if (!spec || !out) return wl::fail(WL_EINVAL, "wl_open_synthetic: spec and out are required");
        *out = nullptr;
        const wl_options o = opt ? *opt : defaults();
        if (in_process_group(o)) {
            wl::Group* g = wl::Group::open(nullptr, spec, o);
            *out = new wl_model{&g->shard(0), g};
            return WL_OK;
        }
        wl::Model* m = wl::Model::open_synthetic(*spec, o);
        *out = new wl_model{m, nullptr};
        return WL_OK;
    });
}

int32_t wl_close(wl_model* model)
{
    return guarded([&]() -> int32_t {
        if (!model) return WL_OK;
        if (model->g) delete model->g;
        else delete model->m;
        delete model;
        return WL_OK;
    });
}

int32_t wl_info_get(const wl_model* model, wl_info* info)
{
    return guarded([&]() -> int32_t {
        if (!model || !info) return wl::fail(WL_EINVAL, "wl_info_get: model and info are required");
        const wl::Config& c = model->m->full_config();
        memset(info, 0, sizeof *info);
        info->layers = c.layers; info->embd = c.embd; info->heads = c.heads; info->kv_heads = c.kv_heads;
        info->head_dim = c.head_dim; info->vocab = c.vocab; info->context_length = c.context_length;
        info->max_context = model->m->max_context(); info->expert_count = c.expert_count;
        info->expert_used = c.expert_used; info->expert_ff = c.expert_ff; info->moe = c.expert_count > 0;
        info->weight_bytes = model->m->weight_bytes(); info->device_bytes = model->m->device_bytes();
        strncpy(info->arch, c.arch.c_str(), sizeof info->arch - 1);
        info->tp_size = model->m->tp_size();
        info->tp_rank = model->g ? -1 : model->m->tp_rank();
        if (model->g)
            for (int g = 1; g < model->g->size(); ++g) info->device_bytes += model->g->shard(g).device_bytes();
        info->tp_fused = model->m->tp_fused() ? 1 : 0;
        return WL_OK;
    });
}

int32_t wl_stats_get(const wl_model* model, wl_stats* stats)
{
    return guarded([&]() -> int32_t {
        if (!model || !stats) return wl::fail(WL_EINVAL, "wl_stats_get: model and stats are required");
        const wl::Stats& s = model->m->stats();
        stats->bytes_h2d = s.bytes_h2d; stats->expert_runs = s.expert_runs; stats->forward_calls = s.forward_calls;
        stats->batch_calls = s.batch_calls; stats->tokens = s.tokens; stats->last_forward_ms = s.last_forward_ms;
        stats->kernel_launches = wl::k::launches() + model->m->graph_launches();
        return WL_OK;
    });
}

int32_t wl_bench_decode(wl_model* model, wl_seq* const* seqs, int32_t N, int32_t steps, double* device_ms)
{
    return guarded([&]() -> int32_t {
        if (!model || !seqs || !device_ms) return wl::fail(WL_EINVAL, "wl_bench_decode: model, seqs and device_ms are required");
        for (int i = 0; i < N; ++i)
            if (!seqs[i] || seqs[i]->owner != model) return wl::fail(WL_EINVAL, "wl_bench_decode: a sequence belongs to another model");
        if (model->g) {
            std::vector<double> ms((size_t)model->g->size(), 0.0);
            model->g->run([&](int g) {
                std::vector<wl::Seq*> ss((size_t)(N > 0 ? N : 0));
                for (int i = 0; i < N; ++i) ss[(size_t)i] = shard_seq(seqs[i], g);
                ms[(size_t)g] = model->g->shard(g).bench_decode(ss.data(), N, steps);
            });
            *device_ms = *std::max_element(ms.begin(), ms.end());
            return WL_OK;
        }
        std::vector<wl::Seq*> ss((size_t)(N > 0 ? N : 0));
        for (int i = 0; i < N; ++i) ss[(size_t)i] = seqs[i]->s;
        *device_ms = model->m->bench_decode(ss.data(), N, steps);
        return WL_OK;
    });
}

int32_t wl_bench_matvecs(wl_model* model, int32_t T, int32_t steps, double* device_ms, double* bytes_per_step)
{
    return guarded([&]() -> int32_t {
        if (!model || !device_ms) return wl::fail(WL_EINVAL, "wl_bench_matvecs: model and device_ms are required");
        if (model->g) {
            std::vector<double> ms((size_t)model->g->size(), 0.0), by((size_t)model->g->size(), 0.0);
            model->g->run([&](int g) { ms[(size_t)g] = model->g->shard(g).bench_matvecs(T, steps, &by[(size_t)g]); });
            *device_ms = *std::max_element(ms.begin(), ms.end());
            if (bytes_per_step) *bytes_per_step = by[0];
            return WL_OK;
        }
        *device_ms = model->m->bench_matvecs(T, steps, bytes_per_step);
        return WL_OK;
    });
}

int32_t wl_profile(wl_model* model, int32_t on)
{
    return guarded([&]() -> int32_t {
        if (!model) return wl::fail(WL_EINVAL, "wl_profile: model is required");
        if (model->g) model->g->run([&](int g) { model->g->shard(g).set_profiling(on != 0); });
        else model->m->set_profiling(on != 0);
        return WL_OK;
    });
}

int32_t wl_profile_get(wl_model* model, int32_t type, wl_profile_entry* out)
{
    return guarded([&]() -> int32_t {
        if (!model || !out) return wl::fail(WL_EINVAL, "wl_profile_get: model and out are required");
        *out = model->m->profile(type);
        return WL_OK;
    });
}

int32_t wl_seq_new(wl_model* model, wl_seq** out)
{
    return guarded([&]() -> int32_t {
        if (!model || !out) return wl::fail(WL_EINVAL, "wl_seq_new: model and out are required");
        wl_seq* q = new wl_seq{model->m->new_seq(), model, {}};
        if (model->g) {
            q->shards.push_back(q->s);
            for (int g = 1; g < model->g->size(); ++g) q->shards.push_back(model->g->shard(g).new_seq());
        }
        *out = q;
        return WL_OK;
    });
}

int32_t wl_seq_free(wl_seq* seq)
{
    return guarded([&]() -> int32_t {
        if (!seq) return WL_OK;
        if (seq->owner->g)
            for (int g = 1; g < seq->owner->g->size(); ++g) seq->owner->g->shard(g).free_seq(seq->shards[(size_t)g]);
        seq->owner->m->free_seq(seq->s);
        delete seq;
        return WL_OK;
    });
}

// Sequence.Truncate (src/Batch.cs:28): drops cached positions from n onward.
int32_t wl_seq_truncate(wl_seq* seq, int32_t n)
{
    return guarded([&]() -> int32_t {
        if (!seq) return wl::fail(WL_EINVAL, "wl_seq_truncate: seq is required");
        if (seq->shards.empty()) {
            if (n < seq->s->length) seq->s->length = n < 0 ? 0 : n;
        } else {
            for (wl::Seq* s : seq->shards)
                if (n < s->length) s->length = n < 0 ? 0 : n;
        }
        return WL_OK;
    });
}

int32_t wl_seq_length(const wl_seq* seq, int32_t* n)
{
    return guarded([&]() -> int32_t {
        if (!seq || !n) return wl::fail(WL_EINVAL, "wl_seq_length: seq and n are required");
        *n = seq->s->length;
        return WL_OK;
    });
}

int32_t wl_truncate(wl_model* model, int32_t n)
{
    return guarded([&]() -> int32_t {
        if (!model) return wl::fail(WL_EINVAL, "wl_truncate: model is required");
        const int G = model->g ? model->g->size() : 1;
        for (int g = 0; g < G; ++g) {
            wl::Seq* s = model->g ? model->g->shard(g).own() : model->m->own();
            if (n < s->length) s->length = n < 0 ? 0 : n;
        }
        return WL_OK;
    });
}

int32_t wl_length(const wl_model* model, int32_t* n)
{
    return guarded([&]() -> int32_t {
        if (!model || !n) return wl::fail(WL_EINVAL, "wl_length: model and n are required");
        *n = model->m->own()->length;
        return WL_OK;
    });
}

namespace {
// wl_forward, wl_forward_argmax and wl_forward_sample: rows come back as logits (logits_out), as their argmax
// (ids_out) or as ids sampled with the options in samp (ids_out and samp).
int32_t forward_rows(const char* fn, wl_model* model, wl_seq* seq, const int32_t* tokens, int32_t T, int32_t pos0,
                     int32_t all_rows, float* logits_out, int32_t* ids_out, volatile const int32_t* cancel,
                     wl_progress_fn progress, void* user, const wl::Model::SampleRows* samp = nullptr)
{
    if (model && T == 0) return wl::fail(WL_EINVAL, "No tokens to run.");
    if (!model || !tokens || !(logits_out || ids_out))
        return wl::fail(WL_EINVAL, std::string(fn) + ": model, tokens and " + (ids_out || !logits_out ? "ids_out" : "logits_out") + " are required");
    if (seq && seq->owner != model) return wl::fail(WL_EINVAL, std::string(fn) + ": the sequence belongs to another model");
    auto call = [&](wl::Model& m, wl::Seq* s, float* out, int32_t* ids, wl_progress_fn pf, void* u) {
        if (ids && samp) return m.forward_sample(s, tokens, T, pos0, *samp, ids, cancel, pf, u);
        return ids ? m.forward_argmax(s, tokens, T, pos0, all_rows != 0, ids, cancel, pf, u)
                   : m.forward(s, tokens, T, pos0, all_rows != 0, out, cancel, pf, u);
    };
    int32_t st;
    if (model->g) {
        // every shard runs the same call; shard 0's results are returned and its thread (the caller) reports
        // progress; the others take the same path (a progress callback that does nothing)
        std::vector<int32_t> sts((size_t)model->g->size(), WL_OK);
        const size_t rows = all_rows ? (size_t)T : 1;
        model->g->run([&](int g) {
            wl::Model& m = model->g->shard(g);
            float* out = nullptr;
            int32_t* ids = nullptr;
            if (g == 0) { out = logits_out; ids = ids_out; }
            else if (ids_out) ids = reinterpret_cast<int32_t*>(model->g->scratch(g, rows));
            else out = model->g->scratch(g, rows * (size_t)m.config().vocab);
            sts[(size_t)g] = call(m, seq ? shard_seq(seq, g) : nullptr, out, ids,
                                  g == 0 ? progress : (progress ? noop_progress : nullptr), g == 0 ? user : nullptr);
        });
        st = sts[0];
    } else {
        st = call(*model->m, seq ? seq->s : nullptr, logits_out, ids_out, progress, user);
    }
    if (st == WL_CANCELLED) return wl::fail(st, "The operation was canceled.");
    return st;
}

int32_t forward_batch_rows(const char* fn, wl_model* model, wl_seq* const* seqs, const int32_t* tokens, int32_t N,
                           float* logits_out, int32_t* ids_out, volatile const int32_t* cancel,
                           wl_progress_fn progress, void* user, const wl::Model::SampleRows* samp = nullptr)
{
    if (!model || !seqs || !tokens || !(logits_out || ids_out))
        return wl::fail(WL_EINVAL, std::string(fn) + ": model, seqs, tokens and " + (ids_out || !logits_out ? "ids_out" : "logits_out") + " are required");
    if (N <= 0) return wl::fail(WL_EINVAL, "ForwardBatch needs one token for each sequence.");
    for (int i = 0; i < N; ++i)
        if (!seqs[i] || seqs[i]->owner != model) return wl::fail(WL_EINVAL, std::string(fn) + ": a sequence belongs to another model");
    auto call = [&](wl::Model& m, wl::Seq* const* ss, float* out, int32_t* ids, wl_progress_fn pf, void* u) {
        if (ids && samp) return m.forward_batch_sample(ss, tokens, N, *samp, ids, cancel, pf, u);
        return ids ? m.forward_batch_argmax(ss, tokens, N, ids, cancel, pf, u)
                   : m.forward_batch(ss, tokens, N, out, cancel, pf, u);
    };
    int32_t st;
    if (model->g) {
        std::vector<int32_t> sts((size_t)model->g->size(), WL_OK);
        model->g->run([&](int g) {
            wl::Model& m = model->g->shard(g);
            std::vector<wl::Seq*> ss((size_t)N);
            for (int i = 0; i < N; ++i) ss[(size_t)i] = shard_seq(seqs[i], g);
            float* out = nullptr;
            int32_t* ids = nullptr;
            if (g == 0) { out = logits_out; ids = ids_out; }
            else if (ids_out) ids = reinterpret_cast<int32_t*>(model->g->scratch(g, (size_t)N));
            else out = model->g->scratch(g, (size_t)N * m.config().vocab);
            sts[(size_t)g] = call(m, ss.data(), out, ids, g == 0 ? progress : (progress ? noop_progress : nullptr),
                                  g == 0 ? user : nullptr);
        });
        st = sts[0];
    } else {
        std::vector<wl::Seq*> ss((size_t)N);
        for (int i = 0; i < N; ++i) ss[(size_t)i] = seqs[i]->s;
        st = call(*model->m, ss.data(), logits_out, ids_out, progress, user);
    }
    if (st == WL_CANCELLED) return wl::fail(st, "The operation was canceled.");
    return st;
}
}  // namespace

int32_t wl_forward(wl_model* model, wl_seq* seq, const int32_t* tokens, int32_t T, int32_t pos0, int32_t all_logits,
                   float* logits_out, volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    return guarded([&]() -> int32_t {
        if (!logits_out && model && T != 0) return wl::fail(WL_EINVAL, "wl_forward: model, tokens and logits_out are required");
        return forward_rows("wl_forward", model, seq, tokens, T, pos0, all_logits, logits_out, nullptr, cancel,
                            progress, user);
    });
}

int32_t wl_forward_argmax(wl_model* model, wl_seq* seq, const int32_t* tokens, int32_t T, int32_t pos0,
                          int32_t all_rows, int32_t* ids_out, volatile const int32_t* cancel, wl_progress_fn progress,
                          void* user)
{
    return guarded([&]() -> int32_t {
        if (!ids_out && model && T != 0) return wl::fail(WL_EINVAL, "wl_forward_argmax: model, tokens and ids_out are required");
        return forward_rows("wl_forward_argmax", model, seq, tokens, T, pos0, all_rows, nullptr, ids_out, cancel,
                            progress, user);
    });
}

int32_t wl_forward_batch(wl_model* model, wl_seq* const* seqs, const int32_t* tokens, int32_t N, float* logits_out,
                         volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    return guarded([&]() -> int32_t {
        if (!logits_out) return wl::fail(WL_EINVAL, "wl_forward_batch: model, seqs, tokens and logits_out are required");
        return forward_batch_rows("wl_forward_batch", model, seqs, tokens, N, logits_out, nullptr, cancel, progress, user);
    });
}

int32_t wl_forward_batch_argmax(wl_model* model, wl_seq* const* seqs, const int32_t* tokens, int32_t N,
                                int32_t* ids_out, volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    return guarded([&]() -> int32_t {
        if (!ids_out) return wl::fail(WL_EINVAL, "wl_forward_batch_argmax: model, seqs, tokens and ids_out are required");
        return forward_batch_rows("wl_forward_batch_argmax", model, seqs, tokens, N, nullptr, ids_out, cancel, progress,
                                  user);
    });
}

int32_t wl_forward_sample(wl_model* model, wl_seq* seq, const int32_t* tokens, int32_t T, int32_t pos0,
                          double temperature, double top_p, double draw, int32_t* id_out,
                          volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    return guarded([&]() -> int32_t {
        if (!id_out && model && T != 0) return wl::fail(WL_EINVAL, "wl_forward_sample: model, tokens and id_out are required");
        if (temperature > 0.0 && !(draw >= 0.0 && draw < 1.0)) return wl::fail(WL_EINVAL, "wl_forward_sample: the draw must be in [0, 1)");
        const wl::Model::SampleRows sr{&temperature, &top_p, &draw};
        return forward_rows("wl_forward_sample", model, seq, tokens, T, pos0, 0, nullptr, id_out, cancel, progress,
                            user, &sr);
    });
}

int32_t wl_forward_batch_sample(wl_model* model, wl_seq* const* seqs, const int32_t* tokens, int32_t N,
                                const double* temperature, const double* top_p, const double* draws, int32_t* ids_out,
                                volatile const int32_t* cancel, wl_progress_fn progress, void* user)
{
    return guarded([&]() -> int32_t {
        if (!ids_out || !temperature || !top_p || !draws)
            return wl::fail(WL_EINVAL, "wl_forward_batch_sample: model, seqs, tokens, temperature, top_p, draws and ids_out are required");
        for (int i = 0; i < N; ++i)
            if (temperature[i] > 0.0 && !(draws[i] >= 0.0 && draws[i] < 1.0))
                return wl::fail(WL_EINVAL, "wl_forward_batch_sample: every draw must be in [0, 1)");
        const wl::Model::SampleRows sr{temperature, top_p, draws};
        return forward_batch_rows("wl_forward_batch_sample", model, seqs, tokens, N, nullptr, ids_out, cancel,
                                  progress, user, &sr);
    });
}

int32_t wl_forward_mixed(wl_model* model, wl_seq* const* seqs, const int32_t* counts, int32_t N, const int32_t* tokens,
                         float* logits_out, int32_t* ids_out, volatile const int32_t* cancel, wl_progress_fn progress,
                         void* user)
{
    return guarded([&]() -> int32_t {
        if (!model || !seqs || !counts || !tokens || (!logits_out && !ids_out))
            return wl::fail(WL_EINVAL, "wl_forward_mixed: model, seqs, counts, tokens and logits_out or ids_out are required");
        if (N <= 0) return wl::fail(WL_EINVAL, "A mixed step needs at least one sequence.");
        for (int i = 0; i < N; ++i)
            if (!seqs[i] || seqs[i]->owner != model) return wl::fail(WL_EINVAL, "wl_forward_mixed: a sequence belongs to another model");
        int32_t st;
        if (model->g) {
            std::vector<int32_t> sts((size_t)model->g->size(), WL_OK);
            model->g->run([&](int g) {
                wl::Model& m = model->g->shard(g);
                std::vector<wl::Seq*> ss((size_t)N);
                for (int i = 0; i < N; ++i) ss[(size_t)i] = shard_seq(seqs[i], g);
                float* out = nullptr;
                int32_t* ids = nullptr;
                if (g == 0) { out = ids_out ? nullptr : logits_out; ids = ids_out; }
                else if (ids_out) ids = reinterpret_cast<int32_t*>(model->g->scratch(g, (size_t)N));
                else out = model->g->scratch(g, (size_t)N * m.config().vocab);
                sts[(size_t)g] = m.forward_mixed(ss.data(), counts, N, tokens, out, ids, cancel,
                                                 g == 0 ? progress : (progress ? noop_progress : nullptr),
                                                 g == 0 ? user : nullptr);
            });
            st = sts[0];
        } else {
            std::vector<wl::Seq*> ss((size_t)N);
            for (int i = 0; i < N; ++i) ss[(size_t)i] = seqs[i]->s;
            st = model->m->forward_mixed(ss.data(), counts, N, tokens, ids_out ? nullptr : logits_out, ids_out, cancel,
                                         progress, user);
        }
        if (st == WL_CANCELLED) return wl::fail(st, "The operation was canceled.");
        return st;
    });
}

int32_t wl_generate_greedy(wl_model* model, wl_seq* seq, int32_t token, int32_t max_new, const int32_t* stop_ids,
                           int32_t n_stop, int32_t chunk, int32_t* ids_out, int32_t* n_out,
                           volatile const int32_t* cancel)
{
    return guarded([&]() -> int32_t {
        if (!model || !n_out || (max_new > 0 && !ids_out))
            return wl::fail(WL_EINVAL, "wl_generate_greedy: model, ids_out and n_out are required");
        if (seq && seq->owner != model) return wl::fail(WL_EINVAL, "wl_generate_greedy: the sequence belongs to another model");
        int32_t st;
        if (model->g) {
            const int G = model->g->size();
            std::vector<int32_t> sts((size_t)G, WL_OK), ns((size_t)G, 0);
            model->g->run([&](int g) {
                wl::Model& m = model->g->shard(g);
                int32_t* ids = g == 0 ? ids_out
                                      : reinterpret_cast<int32_t*>(model->g->scratch(g, (size_t)std::max(max_new, 1)));
                sts[(size_t)g] = m.generate_greedy(seq ? shard_seq(seq, g) : nullptr, token, max_new, stop_ids, n_stop,
                                                   chunk, ids, &ns[(size_t)g], cancel);
            });
            st = sts[0];
            *n_out = ns[0];
        } else {
            st = model->m->generate_greedy(seq ? seq->s : nullptr, token, max_new, stop_ids, n_stop, chunk, ids_out,
                                           n_out, cancel);
        }
        if (st == WL_CANCELLED) return wl::fail(st, "The operation was canceled.");
        return st;
    });
}

int32_t wl_selftest_allreduce_timeout(int32_t device, int32_t wait_ms)
{
    return guarded([&]() -> int32_t {
        if (wait_ms <= 0 || wait_ms > 10000) return wl::fail(WL_EINVAL, "wl_selftest_allreduce_timeout: wait_ms must be 1..10000");
        WL_CUDA(cudaSetDevice(device));
        const int code = wl::k::selftest_ar_wait((long long)wait_ms * 1000000LL);
        if (code == 2) return wl::fail(WL_ETIMEDOUT, "a device-side wait gave up (code 2): a tensor-parallel peer did not arrive");
        return wl::fail(WL_ECUDA, "the all-reduce wait did not give up (code " + std::to_string(code) + ")");
    });
}

int32_t wl_kernel_status(int32_t device)
{
    return guarded([&]() -> int32_t {
        if (device < 0 || device >= 64) return wl::fail(WL_EINVAL, "wl_kernel_status: device ordinal out of range");
        WL_CUDA(cudaSetDevice(device));
        WL_CUDA(cudaDeviceSynchronize());
        int code = 0;
        {
            std::lock_guard<std::mutex> lock(g_scratch_mu);
            code = g_scratch_code[device];
            g_scratch_code[device] = 0;
            if (g_scratch[device]) {
                int e = 0;
                WL_CUDA(cudaMemcpy(&e, g_scratch[device], sizeof e, cudaMemcpyDeviceToHost));
                if (e) {
                    if (!code) code = e;
                    WL_CUDA(cudaMemset(g_scratch[device], 0, sizeof e));
                }
            }
        }
        int e = 0;
        WL_CUDA(cudaMemcpy(&e, wl::k::static_scratch(), sizeof e, cudaMemcpyDeviceToHost));
        if (e) {
            if (!code) code = e;
            WL_CUDA(cudaMemset(wl::k::static_scratch(), 0, sizeof e));
        }
        if (code) return wl::fail(WL_ETIMEDOUT, "a device-side wait of a kernel-level call gave up (code " + std::to_string(code) + ")");
        return WL_OK;
    });
}

int32_t wl_route(const float* dev_logits, int32_t T, int32_t n, int32_t k, int32_t renorm, int32_t* dev_sel,
                 float* dev_wts, void* stream)
{
    return guarded([&]() -> int32_t {
        if (T <= 0 || n <= 0 || n > 256 || k <= 0 || k > 32 || k > n)
            return wl::fail(WL_EINVAL, "wl_route: T >= 1, 1 <= k <= min(n, 32), n <= 256");
        if (!dev_logits || !dev_sel || !dev_wts) return wl::fail(WL_EINVAL, "wl_route: null pointer");
        wl::k::route(dev_logits, T, n, k, renorm, dev_sel, dev_wts, (cudaStream_t)stream);
        WL_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
        return WL_OK;
    });
}

int32_t wl_argmax(const float* dev_logits, int32_t V, int32_t rows, int32_t* dev_ids, void* stream)
{
    return guarded([&]() -> int32_t {
        if (V <= 0 || rows <= 0 || rows > 65535) return wl::fail(WL_EINVAL, "wl_argmax: V and rows must be positive (rows <= 65535)");
        if (!dev_logits || !dev_ids) return wl::fail(WL_EINVAL, "wl_argmax: null pointer");
        const cudaStream_t s = (cudaStream_t)stream;
        void* scratch = nullptr;
        const size_t kb = sizeof(unsigned long long) * (size_t)rows, cb = sizeof(unsigned) * (size_t)rows;
        WL_CUDA(cudaMalloc(&scratch, kb + cb));
        try {
            WL_CUDA(cudaMemsetAsync(scratch, 0, kb + cb, s));
            wl::k::argmax(dev_logits, V, rows, (unsigned long long*)scratch, (unsigned*)((char*)scratch + kb), dev_ids,
                          nullptr, nullptr, s);
            WL_CUDA(cudaStreamSynchronize(s));
        } catch (...) {
            cudaFree(scratch);
            throw;
        }
        WL_CUDA(cudaFree(scratch));
        return WL_OK;
    });
}

int32_t wl_sample(const float* dev_logits, int32_t V, double temperature, double top_p, double draw, int32_t* dev_id,
                  void* stream)
{
    return guarded([&]() -> int32_t {
        if (V <= 0) return wl::fail(WL_EINVAL, "wl_sample: V must be positive");
        if (!dev_logits || !dev_id) return wl::fail(WL_EINVAL, "wl_sample: null pointer");
        if (temperature > 0.0 && !(draw >= 0.0 && draw < 1.0)) return wl::fail(WL_EINVAL, "wl_sample: the draw must be in [0, 1)");
        const cudaStream_t s = (cudaStream_t)stream;
        void* ws = nullptr;
        WL_CUDA(cudaMalloc(&ws, wl::k::sample_workspace_bytes(V)));
        try {
            wl::k::sample_workspace_init(ws, s);
            wl::k::sample(dev_logits, V, temperature, top_p, draw, ws, dev_id, s);
            WL_CUDA(cudaStreamSynchronize(s));
        } catch (...) {
            cudaFree(ws);
            throw;
        }
        WL_CUDA(cudaFree(ws));
        return WL_OK;
    });
}

int32_t wl_dequant(int32_t type, const void* dev_blocks, int64_t n, float* dev_out, void* stream)
{
    return guarded([&]() -> int32_t {
        int b = 0, s = 0;
        if (!wl::can_decode(type) || !wl::layout(type, &b, &s)) return wl::fail(WL_EUNSUPPORTED, "wl_dequant: unsupported type");
        if (n < 0 || n % b != 0) return wl::fail(WL_EINVAL, "wl_dequant: n must be a whole number of blocks");
        if (n > 0 && (!dev_blocks || !dev_out)) return wl::fail(WL_EINVAL, "wl_dequant: null pointer");
        wl::k::init_tables();
        wl::k::dequant(type, dev_blocks, n, dev_out, (cudaStream_t)stream);
        return WL_OK;
    });
}

int32_t wl_matvec(int32_t type, const void* dev_w, int32_t rows, int32_t cols, const float* dev_x, int32_t ncols,
                  float* dev_y, void* stream)
{
    return guarded([&]() -> int32_t {
        int b = 0, s = 0;
        if (!wl::can_decode(type) || !wl::layout(type, &b, &s)) return wl::fail(WL_EUNSUPPORTED, "wl_matvec: unsupported type");
        if (rows <= 0 || cols <= 0 || ncols <= 0 || cols % b != 0) return wl::fail(WL_EINVAL, "MatMul shape mismatch.");
        if (!dev_w || !dev_x || !dev_y) return wl::fail(WL_EINVAL, "wl_matvec: null pointer");
        wl::k::init_tables();
        // every column computed as if alone (MatMulEach): the matvec, never the GEMM
        run_matvec(type, (const uint8_t*)dev_w, rows, cols, dev_x, ncols, dev_y, false, (cudaStream_t)stream, false);
        return WL_OK;
    });
}

// A Q4_K tensor-core matvec with its scratch in a static device array instead of the growing export scratch: nothing
// is allocated here, so callers that own all device memory can use it. The kernel reads the GGUF rows through a TMA
// tensor map (wl_matvec's repacks them into tiles first); both agree within the matvec tolerance.
int32_t wl_matvec_static(int32_t type, const void* dev_w, int32_t rows, int32_t cols, const float* dev_x,
                         int32_t ncols, float* dev_y, void* stream)
{
    return guarded([&]() -> int32_t {
        int b = 0, s = 0;
        if (!wl::can_decode(type) || !wl::layout(type, &b, &s))
            return wl::fail(WL_EUNSUPPORTED, "wl_matvec_static: unsupported type");
        if (rows <= 0 || cols <= 0 || ncols <= 0 || cols % b != 0) return wl::fail(WL_EINVAL, "MatMul shape mismatch.");
        if (!dev_w || !dev_x || !dev_y) return wl::fail(WL_EINVAL, "wl_matvec_static: null pointer");
        if (cols > wl::k::STATIC_MAX_COLS)
            return wl::fail(WL_EINVAL, "wl_matvec_static: cols " + std::to_string(cols) + " exceeds the static scratch limit of " +
                                       std::to_string(wl::k::STATIC_MAX_COLS) + "; use wl_matvec");
        const int64_t rb = wl::row_bytes_of(type, cols);
        if (!wl::k::mma_supported(type, (const uint8_t*)dev_w, rb, cols))
            return wl::fail(WL_EUNSUPPORTED, "wl_matvec_static: only Q4_K weights with 16-byte aligned rows and cols a "
                                             "multiple of 256 have the tensor-core matvec; use wl_matvec");
        if ((uintptr_t)dev_x % 16 != 0) return wl::fail(WL_EINVAL, "wl_matvec_static: dev_x must be 16-byte aligned");
        const size_t need = 256 + wl::k::xprep_bytes(cols, 8);
        if (need > wl::k::STATIC_SCRATCH_BYTES) return wl::fail(WL_EINVAL, "wl_matvec_static: static scratch too small");
        const cudaStream_t st = (cudaStream_t)stream;
        uint8_t* scratch = (uint8_t*)wl::k::static_scratch();
        wl::k::prepare_matvec_mma();        // every column count's kernel attribute, once per device
        int* err = (int*)scratch;
        WL_CUDA(cudaMemsetAsync(scratch + 128, 0, sizeof(int), st));   // orders the launches behind all earlier work
        wl::k::WeightMap map;
        wl::k::make_weight_map(type, (const uint8_t*)dev_w, rows, rb, &map);
        for (int c0 = 0; c0 < ncols; c0 += 8) {
            const int nc = ncols - c0 < 8 ? ncols - c0 : 8;
            const wl::k::XPrep p = wl::k::xprep_view(scratch + 256, cols, nc);
            wl::k::xprep(dev_x + (int64_t)c0 * cols, cols, cols, nc, p, st);
            wl::k::matvec_mma(type, map, 0, rows, cols, p, dev_y + (int64_t)c0 * rows, rows, err, st);
        }
        return WL_OK;
    });
}

int32_t wl_tiles_size(int32_t type, int32_t rows, int32_t cols, int64_t* bytes)
{
    return guarded([&]() -> int32_t {
        if (!bytes) return wl::fail(WL_EINVAL, "wl_tiles_size: bytes is required");
        if (!wl::k::tiles_supported(type, cols)) return wl::fail(WL_EUNSUPPORTED, "wl_tiles_size: no tile layout for this type and width");
        if (rows <= 0) return wl::fail(WL_EINVAL, "MatMul shape mismatch.");
        *bytes = wl::k::tile_bytes(type, rows, cols);
        return WL_OK;
    });
}

int32_t wl_make_tiles(int32_t type, const void* dev_w, int32_t rows, int32_t cols, void* dev_tiles, void* stream)
{
    return guarded([&]() -> int32_t {
        if (!wl::k::tiles_supported(type, cols)) return wl::fail(WL_EUNSUPPORTED, "wl_make_tiles: no tile layout for this type and width");
        if (rows <= 0) return wl::fail(WL_EINVAL, "MatMul shape mismatch.");
        if (!dev_w || !dev_tiles) return wl::fail(WL_EINVAL, "wl_make_tiles: null pointer");
        if ((uintptr_t)dev_tiles % 16 != 0) return wl::fail(WL_EINVAL, "wl_make_tiles: dev_tiles must be 16-byte aligned");
        wl::k::make_tiles(type, (const uint8_t*)dev_w, rows, cols, wl::row_bytes_of(type, cols), (uint8_t*)dev_tiles,
                          (cudaStream_t)stream);
        return WL_OK;
    });
}

int32_t wl_matvec_tiles(int32_t type, const void* dev_tiles, int32_t rows, int32_t cols, const float* dev_x,
                        int32_t ncols, float* dev_y, void* stream)
{
    return guarded([&]() -> int32_t {
        if (!wl::k::tiles_supported(type, cols)) return wl::fail(WL_EUNSUPPORTED, "wl_matvec_tiles: no tile layout for this type and width");
        if (rows <= 0 || ncols <= 0) return wl::fail(WL_EINVAL, "MatMul shape mismatch.");
        if (!dev_tiles || !dev_x || !dev_y) return wl::fail(WL_EINVAL, "wl_matvec_tiles: null pointer");
        if ((uintptr_t)dev_tiles % 16 != 0 || (uintptr_t)dev_x % 16 != 0)
            return wl::fail(WL_EINVAL, "wl_matvec_tiles: dev_tiles and dev_x must be 16-byte aligned");
        const cudaStream_t s = (cudaStream_t)stream;
        uint8_t* scratch = (uint8_t*)export_scratch(256 + wl::k::xprep_bytes(cols, 8));
        int* err = (int*)scratch;
        WL_CUDA(cudaMemsetAsync(scratch + 128, 0, sizeof(int), s));   // orders the launches behind all earlier work
        for (int c0 = 0; c0 < ncols; c0 += 8) {
            const int nc = ncols - c0 < 8 ? ncols - c0 : 8;
            const wl::k::XPrep p = wl::k::xprep_view(scratch + 256, cols, nc);
            wl::k::xprep(dev_x + (int64_t)c0 * cols, cols, cols, nc, p, s);
            wl::k::matvec_tiles(type, (const uint8_t*)dev_tiles, 0, rows, cols, p, dev_y + (int64_t)c0 * rows, rows, err, s);
        }
        return WL_OK;
    });
}

int32_t wl_bench_matvec_tiles(int32_t type, const void* const* dev_tiles, int32_t copies, int32_t rows, int32_t cols,
                              const float* dev_x, int32_t ncols, float* dev_y, int32_t iters, double* device_ms,
                              void* stream)
{
    return guarded([&]() -> int32_t {
        if (!wl::k::tiles_supported(type, cols))
            return wl::fail(WL_EUNSUPPORTED, "wl_bench_matvec_tiles: no tile layout for this type and width");
        if (rows <= 0 || ncols <= 0 || ncols > 8 || copies <= 0 || iters <= 0)
            return wl::fail(WL_EINVAL, "wl_bench_matvec_tiles: rows, copies, iters > 0 and 1 <= ncols <= 8");
        if (!dev_tiles || !dev_x || !dev_y || !device_ms) return wl::fail(WL_EINVAL, "wl_bench_matvec_tiles: null pointer");
        for (int i = 0; i < copies; ++i)
            if (!dev_tiles[i] || (uintptr_t)dev_tiles[i] % 16 != 0)
                return wl::fail(WL_EINVAL, "wl_bench_matvec_tiles: every tile buffer must be 16-byte aligned");
        if ((uintptr_t)dev_x % 16 != 0) return wl::fail(WL_EINVAL, "wl_bench_matvec_tiles: dev_x must be 16-byte aligned");
        const cudaStream_t s = (cudaStream_t)stream;
        uint8_t* scratch = (uint8_t*)export_scratch(256 + wl::k::xprep_bytes(cols, 8));
        int* err = (int*)scratch;
        const wl::k::XPrep p = wl::k::xprep_view(scratch + 256, cols, ncols);
        WL_CUDA(cudaMemsetAsync(scratch + 128, 0, sizeof(int), s));   // orders the launches behind all earlier work
        wl::k::xprep(dev_x, cols, cols, ncols, p, s);
        auto run = [&]() {
            for (int i = 0; i < iters; ++i)
                wl::k::matvec_tiles(type, (const uint8_t*)dev_tiles[i % copies], 0, rows, cols, p, dev_y, rows, err, s);
        };
        run();                          // kernel attributes are set outside the capture
        cudaStream_t cs = nullptr;
        WL_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        cudaGraphExec_t exec = nullptr;
        try {
            cudaEvent_t dep = nullptr;
            WL_CUDA(cudaEventCreateWithFlags(&dep, cudaEventDisableTiming));
            WL_CUDA(cudaEventRecord(dep, s));
            WL_CUDA(cudaStreamWaitEvent(cs, dep, 0));
            cudaEventDestroy(dep);
            cudaGraph_t graph = nullptr;
            const int64_t l0 = wl::k::launches();
            WL_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
            for (int i = 0; i < iters; ++i)
                wl::k::matvec_tiles(type, (const uint8_t*)dev_tiles[i % copies], 0, rows, cols, p, dev_y, rows, err, cs);
            WL_CUDA(cudaStreamEndCapture(cs, &graph));
            wl::k::uncount_launches(wl::k::launches() - l0);
            const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            WL_CUDA(ie);
            WL_CUDA(cudaGraphLaunch(exec, cs));     // warm
            WL_CUDA(cudaEventCreate(&e0));
            WL_CUDA(cudaEventCreate(&e1));
            WL_CUDA(cudaEventRecord(e0, cs));
            WL_CUDA(cudaGraphLaunch(exec, cs));
            WL_CUDA(cudaEventRecord(e1, cs));
            WL_CUDA(cudaEventSynchronize(e1));
            float ms = 0.f;
            WL_CUDA(cudaEventElapsedTime(&ms, e0, e1));
            *device_ms = ms;
        } catch (...) {
            if (exec) cudaGraphExecDestroy(exec);
            if (e0) cudaEventDestroy(e0);
            if (e1) cudaEventDestroy(e1);
            cudaStreamSynchronize(cs);
            cudaStreamDestroy(cs);
            throw;
        }
        cudaGraphExecDestroy(exec);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        WL_CUDA(cudaStreamSynchronize(cs));
        cudaStreamDestroy(cs);
        return WL_OK;
    });
}

int32_t wl_gemm_tiles(int32_t type, const void* dev_tiles, int32_t rows, int32_t cols, const float* dev_x, int32_t T,
                      float* dev_y, void* stream)
{
    return guarded([&]() -> int32_t {
        if (!wl::k::gemm_supported(type, cols)) return wl::fail(WL_EUNSUPPORTED, "wl_gemm_tiles: Q4_K with cols a multiple of 256 only");
        if (rows <= 0 || T <= 0) return wl::fail(WL_EINVAL, "MatMul shape mismatch.");
        if (!dev_tiles || !dev_x || !dev_y) return wl::fail(WL_EINVAL, "wl_gemm_tiles: null pointer");
        if ((uintptr_t)dev_tiles % 16 != 0) return wl::fail(WL_EINVAL, "wl_gemm_tiles: dev_tiles must be 16-byte aligned");
        const cudaStream_t s = (cudaStream_t)stream;
        uint8_t* scratch = (uint8_t*)export_scratch(256 + wl::k::gemm_scratch_bytes(T, cols));
        WL_CUDA(cudaMemsetAsync(scratch + 128, 0, sizeof(int), s));   // orders the launch behind all earlier work
        wl::k::gemm_tiles(type, (const uint8_t*)dev_tiles, 0, rows, cols, dev_x, cols, T, dev_y, rows, scratch + 256,
                          (int*)scratch, s);
        return WL_OK;
    });
}

int32_t wl_matmul(int32_t type, const void* dev_w, int32_t rows, int32_t cols, const float* dev_x, int32_t T,
                  float* dev_y, int32_t path, void* stream)
{
    return guarded([&]() -> int32_t {
        int b = 0, s = 0;
        if (!wl::can_decode(type) || !wl::layout(type, &b, &s)) return wl::fail(WL_EUNSUPPORTED, "wl_matmul: unsupported type");
        if (rows <= 0 || cols <= 0 || T <= 0 || cols % b != 0) return wl::fail(WL_EINVAL, "MatMul shape mismatch.");
        if (!dev_w || !dev_x || !dev_y) return wl::fail(WL_EINVAL, "wl_matmul: null pointer");
        if (path < 0 || path > 2) return wl::fail(WL_EINVAL, "wl_matmul: path must be 0, 1 or 2");
        wl::k::init_tables();
        run_matvec(type, (const uint8_t*)dev_w, rows, cols, dev_x, T, dev_y, path == 1, (cudaStream_t)stream, path != 2);
        return WL_OK;
    });
}

int32_t wl_synth_tensor(int32_t type, uint64_t seed, uint32_t tensor_id, int64_t rows, int64_t cols, float sigma,
                        float offset, void* dev_out, void* stream)
{
    return guarded([&]() -> int32_t {
        if (type != 0 && type != 1 && type != 8 && type != 12 && type != 14) return wl::fail(WL_EUNSUPPORTED, "wl_synth_tensor: type must be F32, F16, Q8_0, Q4_K or Q6_K");
        int b = 0, s = 0;
        wl::layout(type, &b, &s);
        if (rows <= 0 || cols <= 0 || cols % b != 0) return wl::fail(WL_EINVAL, "wl_synth_tensor: bad shape");
        if (!dev_out) return wl::fail(WL_EINVAL, "wl_synth_tensor: null pointer");
        wl::k::synth(type, seed, tensor_id, rows, cols, sigma, offset, (uint8_t*)dev_out, (cudaStream_t)stream);
        return WL_OK;
    });
}

}  // extern "C"
