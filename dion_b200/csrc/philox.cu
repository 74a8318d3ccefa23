// Counter-based normal random numbers: Philox-4x32 with 10 rounds (Salmon,
// Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11),
// followed by the Box-Muller transform. Element i of a stream is a pure
// function of (key, stream, i): every rank, every launch and the CPU oracle
// (dion_b200.ops.philox_normal on CPU tensors) produce the same values for
// the same arguments, independent of any other random-number consumer.
//
// Counter for output block j (4 values): (j_lo, j_hi, stream_lo, stream_hi);
// key: (key_lo, key_hi). Uniforms u = (x + 1) / 2^32 in (0, 1], then
//   z0 = sqrt(-2 ln u0) cos(2 pi u1), z1 = sqrt(-2 ln u0) sin(2 pi u1)
// (and z2, z3 from u2, u3), all scaled by `scale`.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "host_utils.h"

namespace bdion {

namespace {

// round constants of the published Philox-4x32 generator
constexpr uint32_t kPhiloxM0 = 0xD2511F53u, kPhiloxM1 = 0xCD9E8D57u;
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u, kPhiloxW1 = 0xBB67AE85u;

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kPhiloxM0, c.x), lo0 = kPhiloxM0 * c.x;
    const uint32_t hi1 = __umulhi(kPhiloxM1, c.z), lo1 = kPhiloxM1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += kPhiloxW0;
    k.y += kPhiloxW1;
  }
  return c;
}

__device__ __forceinline__ float u01(uint32_t x) { return ((float)x + 1.0f) * 2.3283064365386963e-10f; }

__global__ void philox_normal_kernel(float* __restrict__ out, int64_t n, uint2 key, uint64_t stream, float scale) {
  const int64_t nblk = (n + 3) / 4;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < nblk; j += (int64_t)gridDim.x * blockDim.x) {
    const uint4 r = philox4x32_10(make_uint4((uint32_t)j, (uint32_t)(j >> 32), (uint32_t)stream,
                                             (uint32_t)(stream >> 32)),
                                  key);
    const float ra = sqrtf(-2.f * logf(u01(r.x))), rb = sqrtf(-2.f * logf(u01(r.z)));
    float sa, ca, sb, cb;
    sincosf(6.283185307179586f * u01(r.y), &sa, &ca);
    sincosf(6.283185307179586f * u01(r.w), &sb, &cb);
    const float z[4] = {ra * ca * scale, ra * sa * scale, rb * cb * scale, rb * sb * scale};
    const int64_t base = 4 * j;
    if (base + 3 < n) {
      *reinterpret_cast<float4*>(out + base) = make_float4(z[0], z[1], z[2], z[3]);
    } else {
      for (int u = 0; u < 4 && base + u < n; ++u) out[base + u] = z[u];
    }
  }
}

}  // namespace

// out: contiguous fp32 CUDA tensor (16-byte aligned); key 64-bit, stream 64-bit
void philox_normal(at::Tensor& out, int64_t key, int64_t stream, double scale) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous(),
              "dion_b200 philox_normal: contiguous fp32 CUDA tensor expected");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "dion_b200 philox_normal: 16-byte alignment");
  const int64_t n = out.numel();
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(out.device());
  const uint64_t k = (uint64_t)key;
  const int64_t nblk = (n + 3) / 4;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::min<int64_t>((nblk + 255) / 256, (int64_t)sms * 8);
  philox_normal_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr<float>(), n, make_uint2((uint32_t)k, (uint32_t)(k >> 32)), (uint64_t)stream, (float)scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace bdion
