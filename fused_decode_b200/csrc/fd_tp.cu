// Tensor-parallel exchange over NVLink: the exchange buffers every rank maps
// (CUDA IPC), and the kernel that finishes a tensor-parallel MLP layer.
//
// The down-projection kernel of every rank stores its fp32 block partials
// straight into every rank's exchange buffer as words tagged with the round
// number (tp_publish, fd_stream.cuh).  tp_reduce_kernel then waits -- bounded
// -- for each word's tag, sums the partials in rank order (the same order on
// every rank, so all ranks produce identical bits), adds the residual and
// rounds: out = round(sum_r partial_r + hidden).  This replaces
// an NCCL allreduce plus a residual-add launch; no kernel issues a TMA load
// from peer memory, and nothing uses NVLink multicast.
#include "fd_common.cuh"

#include <cuda_runtime.h>

#include <cstring>

using namespace fd;

namespace {

constexpr uint64_t kTpWaitNs = 2000000000ull;  // bounded flag waits: 2 s

FD_DEV uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct TpReduceArgs {
  char* buf;  // this rank's exchange buffer
  int32_t world, m, m_max;
  int64_t n, data_off;
  const void* res;  // residual [m, n] (contiguous)
  void* out;        // [m, n] (contiguous)
  int* status;
};

// One thread per (row, column): grid (row blocks of 128, m).  The words of
// all ranks are loaded together (one round trip), then any whose tag is not
// yet this round's is re-read, bounded.
template <typename T>
__global__ void __launch_bounds__(kTpBlockRows) tp_reduce_kernel(TpReduceArgs a) {
  // The round number was advanced by the previous round's reduce, which has
  // completed once the down-projection kernel before this one has.
  grid_dep_wait();
  // the next layer's gate/up kernel may be scheduled now: it prefetches its
  // weights and waits for this grid before reading anything it writes
  grid_dep_launch();
  int* seqp = reinterpret_cast<int*>(a.buf);
  int* donep = seqp + 1;
  const int seq = *reinterpret_cast<volatile int*>(seqp);
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kTpBlockRows + threadIdx.x;
  const int col = blockIdx.y;
  if (row < a.n) {
    const uint2* d = reinterpret_cast<const uint2*>(a.buf + a.data_off) +
                     (static_cast<int64_t>((seq & 1) * a.world) * a.m_max + col) * a.n + row;
    const int64_t rank_stride = static_cast<int64_t>(a.m_max) * a.n;
    uint2 v[kMaxTpWorld];
#pragma unroll
    for (int rk = 0; rk < kMaxTpWorld; ++rk)
      if (rk < a.world) v[rk] = ld_tagged_sys(d + rk * rank_stride);
    bool ok = true;
    const uint64_t t0 = gtimer();
#pragma unroll
    for (int rk = 0; rk < kMaxTpWorld; ++rk) {
      if (rk < a.world && ok) {
        while (static_cast<int>(v[rk].y) != seq + 1) {
          if (gtimer() - t0 > kTpWaitNs) {
            atomicOr(a.status, kStatusTpTimeout);
            ok = false;
            break;
          }
          __nanosleep(32);
          v[rk] = ld_tagged_sys(d + rk * rank_stride);
        }
      }
    }
    if (ok) {
      float sum = 0.f;
#pragma unroll
      for (int rk = 0; rk < kMaxTpWorld; ++rk)  // rank order: the same sum on every rank
        if (rk < a.world) sum += __uint_as_float(v[rk].x);
      const int64_t o = col * a.n + row;
      sum += to_f32(static_cast<const T*>(a.res)[o]);
      static_cast<T*>(a.out)[o] = from_f32<T>(sum);
    }
  }
  // The last CTA to finish advances this rank's round number.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(donep, 1) == static_cast<int>(gridDim.x * gridDim.y) - 1) {
      *donep = 0;
      *reinterpret_cast<volatile int*>(seqp) = seq + 1;
    }
  }
}

int from_cuda(cudaError_t e) { return e == cudaSuccess ? FD_OK : FD_ERR_LAUNCH; }

}  // namespace

namespace fd_host {

int tp_reduce_launch(char* buf, int world, int m, int m_max, int64_t n, const void* res, void* out, int dtype,
                     int* status, cudaStream_t st) {
  const TpLayout l = tp_layout(world, m_max, n);
  TpReduceArgs a;
  a.buf = buf;
  a.world = world; a.m = m; a.m_max = m_max;
  a.n = n; a.data_off = l.data_off;
  a.res = res; a.out = out; a.status = status;
  const dim3 grid(static_cast<unsigned>(l.nblk), static_cast<unsigned>(m));
  const cudaError_t e = dtype == FD_BF16 ? launch_pdl(tp_reduce_kernel<__nv_bfloat16>, grid, kTpBlockRows, 0, st, a)
                                         : launch_pdl(tp_reduce_kernel<__half>, grid, kTpBlockRows, 0, st, a);
  return from_cuda(e);
}

}  // namespace fd_host

extern "C" {

size_t fd_tp_exchange_bytes(int32_t world, int32_t m_max, int64_t n) {
  if (world < 1 || world > kMaxTpWorld || m_max < 1 || m_max > 16 || n < 1) return 0;
  return static_cast<size_t>(tp_layout(world, m_max, n).bytes);
}

int fd_tp_exchange_alloc(int32_t world, int32_t m_max, int64_t n, void** buf) {
  if (!buf) return FD_ERR_ARG;
  *buf = nullptr;
  const size_t bytes = fd_tp_exchange_bytes(world, m_max, n);
  if (bytes == 0) return FD_ERR_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return FD_ERR_DEVICE;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return FD_ERR_DEVICE;
  }
  *buf = p;
  return FD_OK;
}

int fd_tp_exchange_free(void* buf) {
  if (!buf) return FD_OK;
  return cudaFree(buf) == cudaSuccess ? FD_OK : FD_ERR_DEVICE;
}

int fd_tp_exchange_handle(void* buf, void* handle) {
  if (!buf || !handle) return FD_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, buf) != cudaSuccess) return FD_ERR_DEVICE;
  std::memcpy(handle, &h, sizeof(h));
  return FD_OK;
}

int fd_tp_exchange_open(const void* handle, void** peer) {
  if (!handle || !peer) return FD_ERR_ARG;
  *peer = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return FD_ERR_DEVICE;
  *peer = p;
  return FD_OK;
}

int fd_tp_exchange_close(void* peer) {
  if (!peer) return FD_OK;
  return cudaIpcCloseMemHandle(peer) == cudaSuccess ? FD_OK : FD_ERR_DEVICE;
}

}  // extern "C"
