// Symmetric peer memory over CUDA IPC, and the small kernels that turn it
// into collectives.
//
// Every rank of a process group allocates one device region of the same size
// (cudaMalloc, zero-filled) and exports its IPC handle; the Python side
// exchanges the handles through the process group and maps each peer's region
// (cudaIpcOpenMemHandle with lazy peer access). Afterwards every rank holds
// the base address of every rank's region, so a kernel can store to (or load
// from) the same offset on any GPU of the node over NVLink / NVSwitch.
//
// Kernels:
//   peer_barrier   : epoch barrier over per-rank flag words; one thread per
//                    peer stores the epoch into that peer's flag slot with
//                    st.release.sys and spins (bounded, globaltimer) on its
//                    own slot. A wait that runs out sets the status word and
//                    returns, so the context stays usable.
//   reduce_slots   : dst = sum_w src[w] in a fixed order (deterministic).
//   push           : copy a local buffer into `nrep` destinations (peer
//                    broadcast for an all-gather whose data is not produced by
//                    a GEMM epilogue).
// No TMA is used here; every peer access is a plain 16-byte load or store.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstring>
#include <tuple>

#include "common.cuh"
#include "host_utils.h"
#include "ptx.cuh"

namespace bdion {

namespace {

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// flags layout in every region: [kMaxRanks] uint32 arrival words, then one
// uint32 epoch counter that only the owning rank touches.
constexpr int kMaxRanks = 64;

__global__ void peer_barrier_kernel(const int64_t* __restrict__ peer_flags, uint32_t* my_flags, int rank, int world,
                                    int* status, uint64_t limit_ns) {
  __shared__ uint32_t epoch;
  if (threadIdx.x == 0) {
    epoch = my_flags[kMaxRanks] + 1;
    my_flags[kMaxRanks] = epoch;
  }
  __syncthreads();
  const int j = threadIdx.x;
  if (j >= world) return;
  __threadfence_system();
  uint32_t* dst = reinterpret_cast<uint32_t*>(peer_flags[j]) + rank;
  st_release_sys_u32(dst, epoch);
  const uint64_t t0 = globaltimer_ns();
  // wrap-safe "flag >= epoch"
  while ((int32_t)(ld_acquire_sys_u32(my_flags + j) - epoch) < 0) {
    if (globaltimer_ns() - t0 > limit_ns) {
      report_status(status, kStatusCommTimeout);
      break;
    }
  }
  __threadfence_system();
}

__global__ void reduce_slots_kernel(const float4* __restrict__ src, float4* __restrict__ dst, int64_t n4, int nslots,
                                    int64_t slot_stride4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = src[i];
    for (int w = 1; w < nslots; ++w) {
      const float4 b = src[i + w * slot_stride4];
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    dst[i] = a;
  }
}

__global__ void push_kernel(const uint4* __restrict__ src, const int64_t* __restrict__ dsts, int nrep, int64_t n16) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = src[i];
    for (int r = 0; r < nrep; ++r) reinterpret_cast<uint4*>(dsts[r])[i] = v;
  }
}

int grid_for(int64_t n, int threads) {
  static int sms = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  int64_t g = (n + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, (int64_t)sms * 8));
}

}  // namespace

// Allocates `bytes` (rounded up to 2 MiB) of zeroed device memory and returns
// (address, 64-byte IPC handle as a CPU uint8 tensor).
std::tuple<int64_t, at::Tensor> symm_create(int64_t bytes) {
  TORCH_CHECK(bytes > 0, "dion_b200 symm: size must be positive");
  const int64_t gran = 2 << 20;
  bytes = (bytes + gran - 1) / gran * gran;
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  at::Tensor t = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  return {reinterpret_cast<int64_t>(p), t};
}

int64_t symm_open(const at::Tensor& handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && handle.scalar_type() == at::kByte,
              "dion_b200 symm: bad IPC handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t peer_ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(peer_ptr))); }

void symm_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

// A tensor view of `numel` elements of `dtype` at address `ptr` on the current
// device (no ownership).
at::Tensor symm_view(int64_t ptr, int64_t numel, int64_t dtype) {
  const auto st = static_cast<at::ScalarType>(dtype);
  const int dev = c10::cuda::current_device();
  return at::from_blob(reinterpret_cast<void*>(ptr), {numel},
                       at::TensorOptions().dtype(st).device(at::kCUDA, dev));
}

// peer_flags: int64 CUDA tensor [world] of the flag-area address in every
// rank's region; my_flags: this rank's flag area (address).
void symm_barrier(const at::Tensor& peer_flags, int64_t my_flags, int64_t rank, int64_t world) {
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "dion_b200 symm: bad rank/world");
  TORCH_CHECK(peer_flags.is_cuda() && peer_flags.scalar_type() == at::kLong && peer_flags.numel() >= world,
              "dion_b200 symm: peer_flags must be an int64 CUDA tensor of world addresses");
  c10::cuda::CUDAGuard guard(peer_flags.device());
  peer_barrier_kernel<<<1, 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      peer_flags.data_ptr<int64_t>(), reinterpret_cast<uint32_t*>(my_flags), (int)rank, (int)world,
      status_device_ptr(), wait_limit_ns());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// src: fp32 [nslots, n] contiguous (slot stride n); dst: fp32 [n].
void symm_reduce_slots(const at::Tensor& src, at::Tensor& dst, int64_t nslots) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kFloat && src.is_contiguous(), "reduce_slots: bad src");
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == at::kFloat && dst.is_contiguous(), "reduce_slots: bad dst");
  const int64_t n = dst.numel();
  TORCH_CHECK(src.numel() >= n * nslots && n % 4 == 0, "reduce_slots: sizes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0,
              "reduce_slots: 16-byte alignment");
  c10::cuda::CUDAGuard guard(src.device());
  const int64_t n4 = n / 4;
  reduce_slots_kernel<<<grid_for(n4, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(src.data_ptr<float>()), reinterpret_cast<float4*>(dst.data_ptr<float>()), n4,
      (int)nslots, n4);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// Copies src (contiguous, nbytes a multiple of 16) to every address in dsts.
void symm_push(const at::Tensor& src, const at::Tensor& dsts) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "push: bad src");
  TORCH_CHECK(dsts.is_cuda() && dsts.scalar_type() == at::kLong, "push: dsts must be an int64 CUDA tensor");
  const int64_t nbytes = src.numel() * src.element_size();
  TORCH_CHECK(nbytes % 16 == 0 && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0, "push: 16-byte sizes");
  c10::cuda::CUDAGuard guard(src.device());
  const int64_t n16 = nbytes / 16;
  push_kernel<<<grid_for(n16, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(src.data_ptr()), dsts.data_ptr<int64_t>(), (int)dsts.numel(), n16);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

int64_t symm_flag_bytes() { return (kMaxRanks + 1) * 4; }

}  // namespace bdion
