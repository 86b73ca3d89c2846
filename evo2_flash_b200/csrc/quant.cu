// Static per-tensor E4M3 activation quantisation for the in_proj GEMM:
//   q = e4m3_rn(clamp(x / sx, -448, 448))
// the rule of fp8_emul.quantize_input (fp8_emul.py:76-78), with the correctly
// rounded fp32 division torch performs (quot_e4m3x2: a reciprocal multiply,
// checked against the rounding ties, __fdiv_rn where it cannot decide).  An
// HBM stream: 16-byte loads of 8 bf16, 8-byte stores of 8 e4m3.
#include "common.cuh"

namespace hb {

constexpr int QUANT_THREADS = 128;
constexpr int QUANT_NV = 4;  // 16-byte vectors per thread in flight per pass

// One block per row (grid-stride over rows).  A pass issues all of a thread's
// loads of the row (up to QUANT_NV vectors) before converting any of them.
__global__ void __launch_bounds__(QUANT_THREADS)
quant_e4m3_kernel(const bf16* __restrict__ x, int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                  int M, int K, const float* __restrict__ scale) {
  pdl_entry();
  const float sx = __ldg(scale);
  const bool fast = quot_divisor_ok(sx);
  const float rsx = __frcp_rn(sx);
  const int vpr = K / 8;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (long long)row * ldx);
    uint2* qr = reinterpret_cast<uint2*>(q + (long long)row * ldq);
    for (int base = 0; base < vpr; base += QUANT_NV * QUANT_THREADS) {
      uint4 raw[QUANT_NV];
#pragma unroll
      for (int i = 0; i < QUANT_NV; ++i) {
        const int v = base + i * QUANT_THREADS + (int)threadIdx.x;
        if (v < vpr) raw[i] = __ldcs(xr + v);
      }
#pragma unroll
      for (int i = 0; i < QUANT_NV; ++i) {
        const int v = base + i * QUANT_THREADS + (int)threadIdx.x;
        if (v >= vpr) continue;
        const bf16* e = reinterpret_cast<const bf16*>(&raw[i]);
        __nv_fp8x2_storage_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          o[k] = quot_e4m3x2(__bfloat162float(e[2 * k]), __bfloat162float(e[2 * k + 1]), sx,
                             rsx, fast);
        qr[v] = *reinterpret_cast<const uint2*>(o);
      }
    }
  }
}

int quant_e4m3_launch(const void* x, int64_t ldx, void* q, int64_t ldq, int M, int K,
                      const float* scale, cudaStream_t st) {
  if (M <= 0 || K <= 0) return HYENA_OK;
  HB_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && ldq % 8 == 0, "quant: K, ldx, ldq must be multiples of 8");
  HB_REQUIRE(aligned16(x) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0, "quant: misaligned pointers");
  const int blocks = M < 148 * 12 ? M : 148 * 12;
  launch_kernel(quant_e4m3_kernel, dim3(blocks), dim3(QUANT_THREADS), 0, st, 0u,
                static_cast<const bf16*>(x), ldx, static_cast<uint8_t*>(q), ldq, M, K, scale);
  return check_launch("quant_e4m3_kernel");
}

}  // namespace hb
