// Static per-tensor E4M3 activation quantisation for the in_proj GEMM:
//   q = e4m3_rn(clamp(x / sx, -448, 448))
// the rule of fp8_emul.quantize_input (fp8_emul.py:76-78), with the correctly
// rounded fp32 division torch performs.  An HBM stream: 16-byte loads of 8 bf16,
// 8-byte stores of 8 e4m3.
#include <cuda_fp8.h>

#include "common.cuh"

namespace hb {

// One block per row (grid-stride over rows), 8 elements per thread per step:
// no 64-bit division in the index arithmetic.
__global__ void __launch_bounds__(256)
quant_e4m3_kernel(const bf16* __restrict__ x, int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                  int M, int K, const float* __restrict__ scale) {
  pdl_entry();
  const float sx = __ldg(scale);
  const int vpr = K / 8;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (long long)row * ldx);
    uint2* qr = reinterpret_cast<uint2*>(q + (long long)row * ldq);
    for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
      const uint4 raw = __ldg(xr + v);
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
      // saturating conversion = clamp to +-448 (NaN stays NaN, as torch's clamp)
      __nv_fp8x2_storage_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = make_float2(__fdiv_rn(__bfloat162float(e[2 * k]), sx),
                                     __fdiv_rn(__bfloat162float(e[2 * k + 1]), sx));
        o[k] = __nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
      }
      qr[v] = *reinterpret_cast<const uint2*>(o);
    }
  }
}

int quant_e4m3_launch(const void* x, int64_t ldx, void* q, int64_t ldq, int M, int K,
                      const float* scale, cudaStream_t st) {
  if (M <= 0 || K <= 0) return HYENA_OK;
  HB_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && ldq % 8 == 0, "quant: K, ldx, ldq must be multiples of 8");
  HB_REQUIRE(aligned16(x) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0, "quant: misaligned pointers");
  const int blocks = M < 148 * 8 ? M : 148 * 8;
  launch_kernel(quant_e4m3_kernel, dim3(blocks), dim3(256), 0, st, 0u, static_cast<const bf16*>(x),
                ldx, static_cast<uint8_t*>(q), ldq, M, K, scale);
  return check_launch("quant_e4m3_kernel");
}

}  // namespace hb
