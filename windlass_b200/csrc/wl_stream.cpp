// Layer streaming (wl_options.resident = 0): LayerStream (src/LayerStream.cs:62-264) re-designed for a GPU. The
// weights of each stage (one per layer, then the output head) live in pinned host memory, already in the layout the
// kernels read (tile-major Q4_K/Q6_K, GGUF rows otherwise); two device slots take turns, stage l running from slot
// l % 2. A copy stream moves stage l+1 into the other slot while stage l computes (LayerStream.StartPrefetch,
// :160-170), each copy waiting on an event recorded after the last kernel that read the slot, and the compute stream
// waits on the copy's event before the stage's first kernel (LayerStream.Acquire/WaitSlot, :130-180). The
// embedding, norm weights and biases stay resident (LayerStream reads embedding rows on demand, :235-254).
#include <algorithm>
#include "wl_common.h"
#include "wl_model.h"

namespace wl {

namespace {
int64_t round256(int64_t b) { return (b + 255) / 256 * 256; }
}  // namespace

// Stage of a GGUF tensor under streaming: its layer for blk.N.*, the head stage for output.weight, -1 (resident) for
// the rest. Vectors are loaded resident by their own path whatever this says.
int Model::stage_of_name(const std::string& name) const
{
    if (name.compare(0, 4, "blk.") == 0) {
        const size_t dot = name.find('.', 4);
        if (dot != std::string::npos) return std::stoi(name.substr(4, dot - 4));
    }
    if (name == "output.weight") return c_.layers;
    return -1;
}

// Device memory for streaming: a staging area the loaders fill with one stage's raw tensors, and the two slots.
// raw_upper and slot_upper bound, per stage, the bytes of its raw tensors and of its laid-out form.
void Model::plan_streaming(const std::vector<int64_t>& raw_upper, const std::vector<int64_t>& slot_upper)
{
    stages_.assign((size_t)c_.layers + 1, Stage{});
    staging_size_ = std::max<int64_t>(256, *std::max_element(raw_upper.begin(), raw_upper.end()));
    slot_bytes_ = std::max<int64_t>(256, *std::max_element(slot_upper.begin(), slot_upper.end()));
    WL_CUDA(cudaMalloc(&staging_, (size_t)staging_size_));
    for (int s = 0; s < 2; ++s) {
        WL_CUDA(cudaMalloc(&slot_[s], (size_t)slot_bytes_));
        WL_CUDA(cudaEventCreateWithFlags(&copied_[s], cudaEventDisableTiming));
        WL_CUDA(cudaEventCreateWithFlags(&freed_[s], cudaEventDisableTiming));
    }
    WL_CUDA(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
}

// Device memory for a weight being loaded: the staging area while a streamed stage loads, else the arena.
uint8_t* Model::weight_alloc(int64_t bytes)
{
    if (!streamed_ || cur_stage_ < 0) return arena_alloc(bytes);
    const int64_t a = round256(bytes);
    if (staging_used_ + a > staging_size_) WL_THROW(WL_ENOMEM, "streaming: a stage does not fit its staging area");
    uint8_t* p = staging_ + staging_used_;
    staging_used_ += a;
    return p;
}

// A stage's weights are all in the staging area: lays them out in slot 0 (tiles where the tensor-core matvec reads
// them, GGUF rows otherwise), copies that to pinned host memory and points the weights at the stage's slot.
void Model::end_stage(int l, const std::vector<Weight*>& ws)
{
    if (!streamed_) return;
    Stage& st = stages_.at((size_t)l);
    if (st.host || !st.ws.empty()) WL_THROW(WL_EINVAL, "streaming: stage " + std::to_string(l) + " was laid out twice");
    int64_t off = 0;
    for (Weight* w : ws) {
        if (!w->present()) continue;
        const int total_rows = w->rows * w->experts;
        const bool tiled = k::tiles_supported(w->type, w->cols) &&
                           (w->experts == 1 || ((w->type == 12 || w->type == 14) && w->rows % 16 == 0));
        const int64_t bytes = tiled ? k::tile_bytes(w->type, total_rows, w->cols) : w->bytes;
        if (off + bytes > slot_bytes_) WL_THROW(WL_ENOMEM, "streaming: a stage does not fit its slot");
        if (tiled) k::make_tiles(w->type, w->d, total_rows, w->cols, w->row_bytes, slot_[0] + off, stream_);
        else WL_CUDA(cudaMemcpyAsync(slot_[0] + off, w->d, (size_t)w->bytes, cudaMemcpyDeviceToDevice, stream_));
        st.ws.push_back(StageWeight{w, off, tiled});
        off += round256(bytes);
    }
    st.bytes = off;
    if (off > 0) {
        WL_CUDA(cudaMallocHost((void**)&st.host, (size_t)off));
        WL_CUDA(cudaMemcpyAsync(st.host, slot_[0], (size_t)off, cudaMemcpyDeviceToHost, stream_));
    }
    WL_CUDA(cudaStreamSynchronize(stream_));
    for (const StageWeight& sw : st.ws) {
        uint8_t* p = slot_[l % 2] + sw.off;
        sw.w->d = p;                         // for tiled weights the raw rows are gone: only the tile path reads them
        sw.w->tiles = sw.tiled ? p : nullptr;
        sw.w->streamed_tiles = sw.tiled;
    }
    staging_used_ = 0;
    slot_stage_[0] = slot_stage_[1] = -1;
}

// After loading: the staging area is no longer needed.
void Model::finish_streaming()
{
    if (!streamed_) return;
    if (staging_) cudaFree(staging_);
    staging_ = nullptr;
    staging_size_ = staging_used_ = 0;
    cur_stage_ = -1;
}

void Model::issue_copy(int l)
{
    const int s = l % 2;
    const Stage& st = stages_[(size_t)l];
    WL_CUDA(cudaStreamWaitEvent(copy_stream_, freed_[s], 0));
    WL_CUDA(cudaMemcpyAsync(slot_[s], st.host, (size_t)st.bytes, cudaMemcpyHostToDevice, copy_stream_));
    WL_CUDA(cudaEventRecord(copied_[s], copy_stream_));
    slot_stage_[s] = l;
    stats_.bytes_h2d += st.bytes;
}

// Before stage l's first kernel: its slot holds it (copied now if the prefetch did not), and the next stage starts
// copying into the other slot once the kernels that last read that slot are done.
void Model::stage_acquire(int l)
{
    if (!streamed_) return;
    const int n = (int)stages_.size(), s = l % 2;
    if (stages_[(size_t)l].bytes > 0) {
        if (slot_stage_[s] != l) issue_copy(l);
        WL_CUDA(cudaStreamWaitEvent(stream_, copied_[s], 0));
    }
    const int nx = (l + 1) % n;
    if (nx % 2 != s && slot_stage_[nx % 2] != nx && stages_[(size_t)nx].bytes > 0) issue_copy(nx);
}

// After stage l's last kernel: its slot may be rewritten once those kernels have run.
void Model::stage_release(int l)
{
    if (!streamed_) return;
    WL_CUDA(cudaEventRecord(freed_[l % 2], stream_));
}

void Model::free_streaming()
{
    if (copy_stream_) cudaStreamSynchronize(copy_stream_);
    for (Stage& st : stages_)
        if (st.host) cudaFreeHost(st.host);
    stages_.clear();
    if (staging_) cudaFree(staging_);
    staging_ = nullptr;
    for (int s = 0; s < 2; ++s) {
        if (slot_[s]) cudaFree(slot_[s]);
        if (copied_[s]) cudaEventDestroy(copied_[s]);
        if (freed_[s]) cudaEventDestroy(freed_[s]);
        slot_[s] = nullptr;
        copied_[s] = freed_[s] = nullptr;
    }
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
    copy_stream_ = nullptr;
}

}  // namespace wl
