// Static per-tensor E4M3 activation quantisation for the in_proj GEMM:
//   q = e4m3_rn(clamp(x / sx, -448, 448))
// the rule of fp8_emul.quantize_input (fp8_emul.py:76-78), with the correctly
// rounded fp32 division torch performs (quot_e4m3x2: a reciprocal multiply,
// checked against the rounding ties, __fdiv_rn where it cannot decide).  An
// HBM stream: 16-byte loads of 8 bf16, 8-byte stores of 8 e4m3.
#include "common.cuh"

namespace hb {

constexpr int QUANT_THREADS = 256;

// One block per row (grid-stride over rows), a thread holding NV 16-byte
// vectors of the row (K <= 16384).  A thread's loads of the next row are
// issued before it converts the current one: two rows per block in flight.
template <int NV>
__global__ void __launch_bounds__(QUANT_THREADS)
quant_e4m3_kernel(const bf16* __restrict__ x, int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                  int M, int K, const float* __restrict__ scale) {
  pdl_entry();
  const float sx = __ldg(scale);
  const bool fast = quot_divisor_ok(sx);
  const float rsx = __frcp_rn(sx);
  const int vpr = K / 8;
  const int tid = (int)threadIdx.x;
  uint4 cur[NV], nxt[NV];
  auto load_row = [&](int row, uint4 (&v)[NV]) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (long long)row * ldx);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = tid + i * QUANT_THREADS;
      if (c < vpr) v[i] = __ldcs(xr + c);
    }
  };
  int row = (int)blockIdx.x;
  if (row < M) load_row(row, cur);
  for (; row < M; row += gridDim.x) {
    const int next = row + (int)gridDim.x;
    if (next < M) load_row(next, nxt);
    uint2* qr = reinterpret_cast<uint2*>(q + (long long)row * ldq);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = tid + i * QUANT_THREADS;
      if (c >= vpr) continue;
      const bf16* e = reinterpret_cast<const bf16*>(&cur[i]);
      __nv_fp8x2_storage_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o[k] = quot_e4m3x2(__bfloat162float(e[2 * k]), __bfloat162float(e[2 * k + 1]), sx, rsx,
                           fast);
      qr[c] = *reinterpret_cast<const uint2*>(o);
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) cur[i] = nxt[i];
  }
}

// One resident wave: blocks = SMs x the blocks of this variant an SM holds.
template <int NV>
static int launch_quant(const bf16* x, int64_t ldx, uint8_t* q, int64_t ldq, int M, int K,
                        const float* scale, cudaStream_t st) {
  static const int per_sm = [] {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, quant_e4m3_kernel<NV>, QUANT_THREADS,
                                                      0) != cudaSuccess || n < 1)
      n = 4;
    return n;
  }();
  const int wave = num_sms() * per_sm;
  const int blocks = M < wave ? M : wave;
  launch_kernel(quant_e4m3_kernel<NV>, dim3(blocks), dim3(QUANT_THREADS), 0, st, 0u, x, ldx, q,
                ldq, M, K, scale);
  return check_launch("quant_e4m3_kernel");
}

int quant_e4m3_launch(const void* x, int64_t ldx, void* q, int64_t ldq, int M, int K,
                      const float* scale, cudaStream_t st) {
  if (M <= 0 || K <= 0) return HYENA_OK;
  HB_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && ldq % 8 == 0, "quant: K, ldx, ldq must be multiples of 8");
  HB_REQUIRE(aligned16(x) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0, "quant: misaligned pointers");
  const int vpr = K / 8;
  const bf16* xb = static_cast<const bf16*>(x);
  uint8_t* qb = static_cast<uint8_t*>(q);
  if (vpr <= 2 * QUANT_THREADS) return launch_quant<2>(xb, ldx, qb, ldq, M, K, scale, st);
  if (vpr <= 4 * QUANT_THREADS) return launch_quant<4>(xb, ldx, qb, ldq, M, K, scale, st);
  if (vpr <= 8 * QUANT_THREADS) return launch_quant<8>(xb, ldx, qb, ldq, M, K, scale, st);
  return fail(HYENA_ERR_UNSUPPORTED, "quant: K above 16384");
}

}  // namespace hb
