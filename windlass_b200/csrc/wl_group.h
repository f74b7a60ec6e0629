// Tensor parallelism inside one process: one wl_model spanning tp_size GPUs (wl_options.tp_rank = -1), for a host
// that runs one process, like the reference's engine (src/Engine.cs). Each GPU holds one rank's shard (a wl::Model,
// devices opt.device .. opt.device + tp_size - 1) and has its own host thread; a call runs every shard's part at once,
// shard 0 on the calling thread (so progress callbacks run there), and returns shard 0's logits (every shard computes
// the same ones).
#pragma once
#include <condition_variable>
#include <exception>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>
#include "wl_model.h"

namespace wl {

class Group {
public:
    // path != nullptr: a GGUF file; else the synthetic spec.
    static Group* open(const char* path, const wl_synth_spec* spec, const wl_options& opt);
    ~Group();
    int size() const { return (int)shards_.size(); }
    Model& shard(int g) { return *shards_[(size_t)g]; }
    // fn(g) for every shard at once, g = 0 on the calling thread; waits for all, then rethrows the first error.
    void run(const std::function<void(int)>& fn);
    // host scratch for the logits of shards 1.. (their copies are not returned)
    float* scratch(int g, size_t floats);

private:
    explicit Group(int G);
    struct Worker {
        std::thread thread;
        std::mutex mu;
        std::condition_variable cv;
        std::function<void()> task;
        bool pending = false, quit = false;
        std::exception_ptr error;
    };
    std::vector<Model*> shards_;
    std::vector<std::unique_ptr<Worker>> workers_;      // workers_[g] serves shard g (index 0 unused)
    std::vector<std::vector<float>> scratch_;
};

}  // namespace wl
