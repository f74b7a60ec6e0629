// In-process tensor parallelism: the shards of one model on several GPUs, one host thread each.
#include "wl_group.h"
#include <cstring>
#include "wl_common.h"
#include "wl_nccl.h"

namespace wl {

Group::Group(int G) : scratch_((size_t)G)
{
    workers_.resize((size_t)G);
    for (int g = 1; g < G; ++g) {
        workers_[(size_t)g].reset(new Worker());
        Worker* w = workers_[(size_t)g].get();
        w->thread = std::thread([w] {
            std::unique_lock<std::mutex> lock(w->mu);
            for (;;) {
                w->cv.wait(lock, [w] { return w->pending || w->quit; });
                if (w->quit) return;
                std::function<void()> task = std::move(w->task);
                lock.unlock();
                std::exception_ptr err;
                try {
                    task();
                } catch (...) {
                    err = std::current_exception();
                }
                lock.lock();
                w->error = err;
                w->pending = false;
                w->cv.notify_all();
            }
        });
    }
}

void Group::run(const std::function<void(int)>& fn)
{
    const int G = (int)workers_.size();
    for (int g = 1; g < G; ++g) {
        Worker* w = workers_[(size_t)g].get();
        std::lock_guard<std::mutex> lock(w->mu);
        w->task = [fn, g] { fn(g); };
        w->error = nullptr;
        w->pending = true;
        w->cv.notify_all();
    }
    std::exception_ptr first;
    try {
        fn(0);
    } catch (...) {
        first = std::current_exception();
    }
    for (int g = 1; g < G; ++g) {
        Worker* w = workers_[(size_t)g].get();
        std::unique_lock<std::mutex> lock(w->mu);
        w->cv.wait(lock, [w] { return !w->pending; });
        if (!first && w->error) first = w->error;
    }
    if (first) std::rethrow_exception(first);
}

float* Group::scratch(int g, size_t floats)
{
    std::vector<float>& v = scratch_[(size_t)g];
    if (v.size() < floats) v.resize(floats);
    return v.data();
}

Group* Group::open(const char* path, const wl_synth_spec* spec, const wl_options& opt)
{
    const int G = opt.tp_size;
    if (G < 2 || G > 64) WL_THROW(WL_EINVAL, "tp_size must be 2 or more for a model spanning several GPUs.");
    int count = 0;
    WL_CUDA(cudaGetDeviceCount(&count));
    if (opt.device < 0 || opt.device + G > count)
        WL_THROW(WL_EINVAL, "Tensor parallelism over " + std::to_string(G) + " GPUs from device " +
                            std::to_string(opt.device) + " needs devices up to " + std::to_string(opt.device + G - 1) +
                            "; " + std::to_string(count) + " are visible.");
    uint8_t id[TP_ID_BYTES];
    Comm::unique_id(id);
    std::unique_ptr<Group> grp(new Group(G));
    std::vector<Model*> models((size_t)G, nullptr);
    try {
        // every shard joins the NCCL group while the others do (ncclCommInitRank blocks until all have joined)
        grp->run([&](int g) {
            wl_options o = opt;
            o.tp_rank = g;
            o.device = opt.device + g;
            memcpy(o.tp_id, id, TP_ID_BYTES);
            models[(size_t)g] = path ? Model::open_file(path, o) : Model::open_synthetic(*spec, o);
        });
    } catch (...) {
        // the shards that did open leave without the collectives of an orderly close: a failed shard is gone
        try {
            grp->run([&](int g) {
                if (models[(size_t)g]) models[(size_t)g]->detach_group();
                delete models[(size_t)g];
            });
        } catch (...) {
        }
        throw;
    }
    grp->shards_ = models;
    return grp.release();
}

Group::~Group()
{
    if (!shards_.empty()) {
        try {
            run([this](int g) {
                delete shards_[(size_t)g];
                shards_[(size_t)g] = nullptr;
            });
        } catch (...) {
        }
    }
    for (size_t g = 1; g < workers_.size(); ++g) {
        Worker* w = workers_[g].get();
        {
            std::lock_guard<std::mutex> lock(w->mu);
            w->quit = true;
            w->cv.notify_all();
        }
        w->thread.join();
    }
}

}  // namespace wl
