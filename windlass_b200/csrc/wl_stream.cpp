// Layer streaming (wl_options.resident = 0): LayerStream (src/LayerStream.cs:62-264) re-designed for a GPU. The
// weights of each stage (one per layer, then the output head) live in pinned host memory, already in the layout the
// kernels read (tile-major Q4_K/Q6_K, GGUF rows otherwise); two device slots take turns, stage l running from slot
// l % 2. A copy stream moves stage l+1 into the other slot while stage l computes (LayerStream.StartPrefetch,
// :160-170), each copy waiting on an event recorded after the last kernel that read the slot, and the compute stream
// waits on the copy's event before the stage's first kernel (LayerStream.Acquire/WaitSlot, :130-180). The
// embedding, norm weights and biases stay resident (LayerStream reads embedding rows on demand, :235-254).
//
// With wl_options.stream_file = 1 no stage is kept in host memory: a reader thread reads each stage's tensors from the
// GGUF file when the stage is next needed (LayerStream's per-stage file reads, :182-232), in 8 MB chunks (the
// reference's chunk size) through a ring of four pinned buffers, with O_DIRECT where the file system takes it, and
// queues each chunk's copy on the copy stream as soon as it is read, so reading and copying overlap; Q4_K/Q6_K and the
// other tiled formats land in the staging area and are repacked into the slot by the tile kernels on the copy stream.
#include <algorithm>
#include <cerrno>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <mutex>
#include <thread>
#include <fcntl.h>
#include <unistd.h>
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
        if (stream_file_) {
            const int64_t raw = (int64_t)(w->d - staging_);
            const auto it = std::find_if(file_src_.begin(), file_src_.end(),
                                         [&](const std::pair<int64_t, std::pair<int64_t, int64_t>>& r) { return r.first == raw; });
            if (it == file_src_.end() || it->second.second != w->bytes)
                WL_THROW(WL_EINVAL, "streaming: a weight of stage " + std::to_string(l) + " has no file range");
            st.file.push_back(FileItem{it->second.first, w->bytes, raw, off, w, tiled, total_rows});
        }
        off += round256(bytes);
    }
    st.bytes = off;
    file_src_.clear();
    if (off > 0 && !stream_file_) {
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

// The reader of file-backed streaming: jobs are stage indices; for each it queues, on the copy stream, the wait for
// the slot, every chunk's copy and the repacks, then the slot's copied event, and reports the stage as queued.
struct Model::FileReader {
    static constexpr int NBUF = 4;
    static constexpr int64_t CHUNK = 8 << 20, ALIGN = 4096;
    int fd = -1;
    bool direct = false;
    uint8_t* buf[NBUF] = {};
    cudaEvent_t ev[NBUF] = {};
    int next = 0;
    std::thread th;
    std::mutex mu;
    std::condition_variable cv;
    std::deque<int> jobs;
    int queued[2] = {-1, -1};           // per slot: the last stage whose copies are queued
    int64_t seq[2] = {0, 0};            // per slot: jobs queued so far (a stage may come round again)
    int64_t want[2] = {0, 0};           // per slot: jobs posted so far
    bool stop = false;
    std::string error;
};

namespace {
// Reads [off, off + n) of fd into p (n bytes), retrying short reads; false at end of file or on an error (errno).
bool read_all(int fd, uint8_t* p, int64_t n, int64_t off, int64_t* got)
{
    int64_t done = 0;
    while (done < n) {
        const ssize_t r = pread(fd, p + done, (size_t)(n - done), (off_t)(off + done));
        if (r < 0) {
            if (errno == EINTR) continue;
            *got = done;
            return false;
        }
        if (r == 0) break;
        done += r;
    }
    *got = done;
    return true;
}
}  // namespace

// Copies the file bytes [off, off + n) to device memory dst through the pinned ring, queued on the copy stream.
void Model::reader_fetch(int l)
{
    FileReader& R = *reader_;
    const int s = l % 2;
    const Stage& st = stages_[(size_t)l];
    WL_CUDA(cudaStreamWaitEvent(copy_stream_, freed_[s], 0));
    for (const FileItem& it : st.file) {
        uint8_t* dst = it.tiled ? staging_ + it.raw_off : slot_[s] + it.slot_off;
        int64_t pos = it.file_off;
        const int64_t end = it.file_off + it.bytes;
        while (pos < end) {
            const int b = R.next;
            R.next = (R.next + 1) % FileReader::NBUF;
            WL_CUDA(cudaEventSynchronize(R.ev[b]));         // the buffer's previous copy has been done
            const int64_t a0 = R.direct ? pos / FileReader::ALIGN * FileReader::ALIGN : pos;
            const int64_t stop = std::min(end, a0 + FileReader::CHUNK);
            const int64_t a1 = R.direct ? (stop + FileReader::ALIGN - 1) / FileReader::ALIGN * FileReader::ALIGN : stop;
            int64_t got = 0;
            const bool ok = read_all(R.fd, R.buf[b], a1 - a0, a0, &got);
            if (!ok || got < stop - a0)
                WL_THROW(WL_EIO, "streaming: reading " + file_path_ + " at " + std::to_string(a0) + " failed" +
                                     (ok ? std::string(" (end of file)") : std::string(": ") + strerror(errno)));
            WL_CUDA(cudaMemcpyAsync(dst + (pos - it.file_off), R.buf[b] + (pos - a0), (size_t)(stop - pos),
                                    cudaMemcpyHostToDevice, copy_stream_));
            WL_CUDA(cudaEventRecord(R.ev[b], copy_stream_));
            pos = stop;
        }
        if (it.tiled)
            k::make_tiles(it.w->type, staging_ + it.raw_off, it.rows_total, it.w->cols, it.w->row_bytes,
                          slot_[s] + it.slot_off, copy_stream_);
    }
    WL_CUDA(cudaEventRecord(copied_[s], copy_stream_));
}

void Model::reader_loop()
{
    FileReader& R = *reader_;
    cudaSetDevice(device_);
    for (;;) {
        int l;
        {
            std::unique_lock<std::mutex> lock(R.mu);
            R.cv.wait(lock, [&] { return R.stop || !R.jobs.empty(); });
            if (R.stop) return;
            l = R.jobs.front();
        }
        std::string err;
        try {
            reader_fetch(l);
        } catch (const Error& e) {
            err = e.msg.empty() ? std::string("streaming: the reader failed") : e.msg;
        } catch (const std::exception& e) {
            err = e.what();
        }
        std::lock_guard<std::mutex> lock(R.mu);
        R.jobs.pop_front();
        R.queued[l % 2] = l;
        ++R.seq[l % 2];
        if (!err.empty() && R.error.empty()) R.error = err;
        R.cv.notify_all();
    }
}

// Blocks until the reader has queued stage l's copies (so its copied event is the one to wait on).
void Model::reader_wait(int l)
{
    FileReader& R = *reader_;
    std::unique_lock<std::mutex> lock(R.mu);
    const int s = l % 2;
    R.cv.wait(lock, [&] { return R.seq[s] >= R.want[s] || !R.error.empty(); });
    if (!R.error.empty()) WL_THROW(WL_EIO, R.error);
    (void)l;
}

// After loading: the staging area is no longer needed (file-backed streaming keeps it for the raw tensors, and
// starts its reader).
void Model::finish_streaming()
{
    if (!streamed_) return;
    cur_stage_ = -1;
    if (stream_file_) {
        reader_ = new FileReader();
        FileReader& R = *reader_;
        R.fd = open(file_path_.c_str(), O_RDONLY | O_DIRECT);
        R.direct = R.fd >= 0;
        if (R.fd < 0) R.fd = open(file_path_.c_str(), O_RDONLY);
        if (R.fd < 0) WL_THROW(WL_EIO, "streaming: cannot open " + file_path_ + ": " + strerror(errno));
        for (int b = 0; b < FileReader::NBUF; ++b) {
            WL_CUDA(cudaMallocHost((void**)&R.buf[b], (size_t)(FileReader::CHUNK + 2 * FileReader::ALIGN)));
            WL_CUDA(cudaEventCreateWithFlags(&R.ev[b], cudaEventDisableTiming));
        }
        // a probe read: some file systems accept O_DIRECT at open and refuse it at read time
        if (R.direct) {
            int64_t got = 0;
            if (!read_all(R.fd, R.buf[0], FileReader::ALIGN, 0, &got)) {
                close(R.fd);
                R.direct = false;
                R.fd = open(file_path_.c_str(), O_RDONLY);
                if (R.fd < 0) WL_THROW(WL_EIO, "streaming: cannot open " + file_path_ + ": " + strerror(errno));
            }
        }
        R.th = std::thread([this] { reader_loop(); });
        return;
    }
    if (staging_) cudaFree(staging_);
    staging_ = nullptr;
    staging_size_ = staging_used_ = 0;
}

void Model::issue_copy(int l)
{
    const int s = l % 2;
    const Stage& st = stages_[(size_t)l];
    slot_stage_[s] = l;
    if (stream_file_) {
        FileReader& R = *reader_;
        std::lock_guard<std::mutex> lock(R.mu);
        R.jobs.push_back(l);
        ++R.want[s];
        R.cv.notify_all();
        int64_t b = 0;
        for (const FileItem& it : st.file) b += it.bytes;
        stats_.bytes_h2d += b;
        return;
    }
    WL_CUDA(cudaStreamWaitEvent(copy_stream_, freed_[s], 0));
    WL_CUDA(cudaMemcpyAsync(slot_[s], st.host, (size_t)st.bytes, cudaMemcpyHostToDevice, copy_stream_));
    WL_CUDA(cudaEventRecord(copied_[s], copy_stream_));
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
        if (stream_file_) reader_wait(l);
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
    if (reader_) {
        FileReader& R = *reader_;
        {
            std::lock_guard<std::mutex> lock(R.mu);
            R.stop = true;
            R.cv.notify_all();
        }
        if (R.th.joinable()) R.th.join();
        if (copy_stream_) cudaStreamSynchronize(copy_stream_);
        for (int b = 0; b < FileReader::NBUF; ++b) {
            if (R.buf[b]) cudaFreeHost(R.buf[b]);
            if (R.ev[b]) cudaEventDestroy(R.ev[b]);
        }
        if (R.fd >= 0) close(R.fd);
        delete reader_;
        reader_ = nullptr;
    }
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
