// NCCL for the tensor-parallel decoder, loaded at run time (dlopen of libnccl.so.2) so that the library loads and
// runs one-GPU models on a machine without NCCL. In a process that already loaded NCCL (PyTorch does), the loaded copy
// is reused; a process that also uses PyTorch should import it before the first tensor-parallel call, since the
// system NCCL loaded first would then be the one PyTorch binds to. WL_NCCL_LIBRARY names another NCCL to load.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace wl {

constexpr int TP_ID_BYTES = 128;     // NCCL_UNIQUE_ID_BYTES

// One rank's handle on a tensor-parallel group: `size` ranks, one GPU each.
class Comm {
public:
    // A fresh group id (ncclGetUniqueId); one rank makes it and every rank passes the same bytes to the constructor.
    static void unique_id(uint8_t out[TP_ID_BYTES]);
    // Joins the group on the current device; blocks until all `size` ranks have joined.
    Comm(const uint8_t id[TP_ID_BYTES], int size, int rank);
    ~Comm();
    Comm(const Comm&) = delete;
    Comm& operator=(const Comm&) = delete;

    // buf[0..n) = the sum over ranks of every rank's buf, in place, on stream s (capturable into a CUDA graph).
    void allreduce_sum(float* buf, int64_t n, cudaStream_t s);
    // buf[0..n) = the maximum over ranks, in place, on stream s.
    void allreduce_max(int32_t* buf, int64_t n, cudaStream_t s);
    // recv[r*n .. (r+1)*n) = rank r's send[0..n), on stream s.
    void allgather(const void* send, void* recv, int64_t bytes_per_rank, cudaStream_t s);

    const int size, rank;

private:
    void* comm_ = nullptr;
};

}  // namespace wl
