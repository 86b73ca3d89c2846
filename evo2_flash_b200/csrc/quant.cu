// Static per-tensor E4M3 activation quantisation for the in_proj GEMM:
//   q = e4m3_rn(clamp(x / sx, -448, 448))
// the rule of fp8_emul.quantize_input (fp8_emul.py:76-78).  A pure HBM stream:
// 16-byte loads of 8 bf16, 8-byte stores of 8 e4m3.
#include <cuda_fp8.h>

#include "common.cuh"

namespace hb {

__global__ void __launch_bounds__(256)
quant_e4m3_kernel(const bf16* __restrict__ x, int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                  int M, int K, const float* __restrict__ scale) {
  pdl_entry();
  const float sx = __ldg(scale);
  const int vpr = K / 8;
  const long long total = (long long)M * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / vpr;
    const int v = int(i % vpr);
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + row * ldx) + v);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
    uint8_t o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float f = __fdiv_rn(__bfloat162float(e[k]), sx);
      f = fminf(fmaxf(f, -448.0f), 448.0f);
      o[k] = __nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3);
    }
    *reinterpret_cast<uint2*>(q + row * ldq + 8 * v) = *reinterpret_cast<const uint2*>(o);
  }
}

int quant_e4m3_launch(const void* x, int64_t ldx, void* q, int64_t ldq, int M, int K,
                      const float* scale, cudaStream_t st) {
  if (M <= 0 || K <= 0) return HYENA_OK;
  HB_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && ldq % 8 == 0, "quant: K, ldx, ldq must be multiples of 8");
  HB_REQUIRE(aligned16(x) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0, "quant: misaligned pointers");
  const long long total = (long long)M * (K / 8);
  long long nb = (total + 255) / 256;
  if (nb > 148LL * 16) nb = 148LL * 16;
  const int blocks = (int)nb;
  launch_kernel(quant_e4m3_kernel, dim3(blocks), dim3(256), 0, st, 0u, static_cast<const bf16*>(x), ldx,
                                            static_cast<uint8_t*>(q), ldq, M, K, scale);
  return check_launch("quant_e4m3_kernel");
}

}  // namespace hb
