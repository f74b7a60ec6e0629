// Sampling on the device: Sampler.Sample of the reference (src/Engine.cs:361-380) for one row of logits, with the
// host's uniform draw (its Random.NextDouble()) passed in, so that a sampled decode step sends back one id instead
// of V floats.
//
//   temperature <= 0: the greedy id (lowest index of the largest logit).
//   p[i] = exp((logit[i] - max) / temperature) in double, max the largest logit.
//   top_p >= 1: r = draw * sum(p); the first i at which the running sum of p in index order reaches r.
//   top_p < 1: order the ids by p descending; the nucleus is the shortest prefix whose running sum reaches
//              top_p * sum(p); pick = draw * (that prefix's sum); the first id of the prefix at which its running sum
//              reaches pick.
//
// The sums are prefix sums (CUB's device scan, a fixed tree) where the reference adds one term at a time, and the
// descending order is CUB's stable radix sort, so equal probabilities keep ascending ids where the reference's
// Array.Sort (an unstable introsort) leaves them in an order of its own. Both change a choice only when a draw
// falls within a few units in the last place of a boundary between two ids, or among exactly equal probabilities.
#include <cstdint>
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>
#include "wl_common.h"
#include "wl_kernels.h"
#include "wl_launch.cuh"

namespace wl {
namespace k {

namespace {

// p[i] = exp((x[i] - x[best]) / temperature) (float difference, as the reference's float arithmetic gives it, then
// the double division and exponential); ids[i] = i. The first thread also resets the nucleus to every id (V - 1, the
// reference's k = n when no prefix reaches the limit) and the crossing position to "none".
__global__ void k_samp_prob(const float* x, int V, const int32_t* best, double temperature,
                            double* p, int32_t* ids, int32_t* nucleus,
                            int32_t* pos)
{
    pdl_trigger();
    pdl_wait();
    const float mx = x[*best];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        *nucleus = V - 1;
        *pos = INT32_MAX;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        p[i] = exp((double)__fsub_rn(x[i], mx) / temperature);
        ids[i] = i;
    }
}

// *out = min(*out, the first position j of the prefix-sum array pre[0..n) with pre[j] >= target). target =
// scale * *total, or, with nucleus, the array is cut after the nucleus's last position and target = scale * pre[that
// position]. The minimum (an atomic one over the positions where the running sum crosses the target) keeps the
// answer the first crossing even where a tree-ordered prefix sum steps down by a unit in the last place over a zero
// term.
__global__ void k_samp_cross(const double* pre, int n, const int32_t* nucleus,
                             const double* total, double scale, int32_t* out)
{
    pdl_trigger();
    pdl_wait();
    if (nucleus) n = *nucleus + 1;
    const double target = scale * (nucleus ? pre[n - 1] : *total);
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        if (pre[j] >= target && (j == 0 || pre[j - 1] < target)) atomicMin(out, j);
    }
}

// The chosen id: ids[*pos] (or *pos itself in index order), and where no position crossed, the reference's fallback:
// the first id of the nucleus (ids[0]) or, in index order, the greedy id.
__global__ void k_samp_final(const int32_t* pos, const int32_t* ids,
                             const int32_t* best, int32_t* out)
{
    pdl_trigger();
    pdl_wait();
    const int32_t j = *pos;
    if (j == INT32_MAX) *out = ids ? ids[0] : *best;
    else *out = ids ? ids[j] : j;
}

}  // namespace

namespace {

// Workspace of one sampled row of V logits: [argmax key u64 | argmax count u32 | best, nucleus, pos i32 | pad to 256]
// then p, sorted p, index-order prefix, sorted prefix (V doubles each), ids, sorted ids (V int32 each), CUB's temp.
struct SampleWs {
    unsigned long long* key;
    unsigned* count;
    int32_t *best, *nucleus, *pos;
    double *p, *ps, *pre, *cum;
    int32_t *ids, *ids_s;
    void* temp;
    size_t temp_bytes;
};

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

size_t cub_temp_bytes(int V)
{
    size_t a = 0, b = 0;
    WL_CUDA(cub::DeviceRadixSort::SortPairsDescending(nullptr, a, (const double*)nullptr, (double*)nullptr,
                                                      (const int32_t*)nullptr, (int32_t*)nullptr, V));
    WL_CUDA(cub::DeviceScan::InclusiveSum(nullptr, b, (const double*)nullptr, (double*)nullptr, V));
    return a > b ? a : b;
}

SampleWs carve(void* ws, int V)
{
    uint8_t* b = (uint8_t*)ws;
    SampleWs w;
    w.key = (unsigned long long*)b;
    w.count = (unsigned*)(b + 8);
    w.best = (int32_t*)(b + 16);
    w.nucleus = (int32_t*)(b + 20);
    w.pos = (int32_t*)(b + 24);
    size_t o = 256;
    w.p = (double*)(b + o); o += align256(8 * (size_t)V);
    w.ps = (double*)(b + o); o += align256(8 * (size_t)V);
    w.pre = (double*)(b + o); o += align256(8 * (size_t)V);
    w.cum = (double*)(b + o); o += align256(8 * (size_t)V);
    w.ids = (int32_t*)(b + o); o += align256(4 * (size_t)V);
    w.ids_s = (int32_t*)(b + o); o += align256(4 * (size_t)V);
    w.temp = b + o;
    w.temp_bytes = cub_temp_bytes(V);
    return w;
}

}  // namespace

size_t sample_workspace_bytes(int V)
{
    return 256 + 4 * align256(8 * (size_t)V) + 2 * align256(4 * (size_t)V) + align256(cub_temp_bytes(V));
}

void sample_workspace_init(void* ws, cudaStream_t s)
{
    WL_CUDA(cudaMemsetAsync(ws, 0, 256, s));      // the argmax key and counter start (and stay) at zero
}

void sample(const float* logits, int V, double temperature, double top_p, double draw, void* ws, int32_t* out_id,
            cudaStream_t s)
{
    if (V <= 0 || !logits || !ws || !out_id) WL_THROW(WL_EINVAL, "sample: V > 0 and the pointers are required");
    const SampleWs w = carve(ws, V);
    // the greedy id: Sampler.Sample's first loop (the lowest index of the largest logit)
    if (!(temperature > 0.0)) {
        argmax(logits, V, 1, w.key, w.count, out_id, nullptr, nullptr, s);
        return;
    }
    if (!(draw >= 0.0 && draw < 1.0)) WL_THROW(WL_EINVAL, "sample: the draw must be in [0, 1)");
    argmax(logits, V, 1, w.key, w.count, w.best, nullptr, nullptr, s);
    const int grid = (V + 255) / 256 < 4 * 148 ? (V + 255) / 256 : 4 * 148;
    launch(k_samp_prob, dim3(grid), dim3(256), 0, s, logits, V, (const int32_t*)w.best, temperature, w.p, w.ids,
           w.nucleus, w.pos);
    note_launch();
    size_t tb = w.temp_bytes;
    WL_CUDA(cub::DeviceScan::InclusiveSum(w.temp, tb, (const double*)w.p, w.pre, V, s));
    const double* sum = w.pre + (V - 1);      // the reference's sum, in index order
    const int32_t* ids = nullptr;
    if (top_p >= 1.0) {
        // r = draw * sum; the first i at which the running sum reaches r
        launch(k_samp_cross, dim3(grid), dim3(256), 0, s, (const double*)w.pre, V, (const int32_t*)nullptr, sum, draw,
               w.pos);
        note_launch();
    } else {
        tb = w.temp_bytes;
        WL_CUDA(cub::DeviceRadixSort::SortPairsDescending(w.temp, tb, (const double*)w.p, w.ps,
                                                          (const int32_t*)w.ids, w.ids_s, V, 0, 64, s));
        tb = w.temp_bytes;
        WL_CUDA(cub::DeviceScan::InclusiveSum(w.temp, tb, (const double*)w.ps, w.cum, V, s));
        // the nucleus: the first sorted position whose running sum reaches top_p * sum (else every id)
        launch(k_samp_cross, dim3(grid), dim3(256), 0, s, (const double*)w.cum, V, (const int32_t*)nullptr, sum,
               top_p, w.nucleus);
        note_launch();
        // pick = draw * (the nucleus's sum); the first sorted position at which the running sum reaches it
        launch(k_samp_cross, dim3(grid), dim3(256), 0, s, (const double*)w.cum, V, (const int32_t*)w.nucleus,
               (const double*)nullptr, draw, w.pos);
        note_launch();
        ids = w.ids_s;
    }
    launch(k_samp_final, dim3(1), dim3(32), 0, s, (const int32_t*)w.pos, ids, (const int32_t*)w.best, out_id);
    note_launch();
}

}  // namespace k
}  // namespace wl
