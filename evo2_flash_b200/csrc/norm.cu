// The decoder layer's Evo2RMSNorm with the residual add and the in_proj input
// quantisation fused in (evo2_flash/model.py:47-76 Evo2RMSNorm, whose CUDA
// form is triton_norm.py:127-156 rms_norm; fp8_emul.py:76-78 for q):
//
//   s = bf16(x + r)                              (r optional; s stored if asked)
//   n = bf16(sqrt(sum_j s_j^2))                  fp32 sum of squares
//   n = bf16(n * H^-0.5);  n = bf16(n + eps)     eps outside the square root
//   y = bf16(w * bf16(s / n))                    (stored if asked)
//   q = e4m3(clamp(y / sx, +-448))               (stored if asked)
//
// every rounding point of the torch code.  The sum of squares runs in this
// kernel's own order (squares of bf16 values are exact in fp32; only the order
// of the fp32 additions differs from ATen's), so n can differ from the
// reference's in its last bf16 bit on rare rows.
//
// One row per CTA pass, 128 threads; a thread holds NV 16-byte vectors of the
// row (vector v = thread + i * 128) from the load to the stores, so the row is
// read once: one HBM pass reads x (and r) and writes only what is asked for
// (the weight vector stays in L1).
#include "common.cuh"

namespace hb {

constexpr int NORM_THREADS = 128;

__device__ __forceinline__ float2 bf2f(uint32_t v) { return unpack2(as_bf162(v)); }

template <int NV>
__global__ void __launch_bounds__(NORM_THREADS) rms_norm_kernel(const NormArgs A) {
  pdl_entry();
  __shared__ float red[2][NORM_THREADS / 32];
  const int tid = (int)threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vpr = A.H / 8;
  const float sx = A.q != nullptr ? __ldg(A.sx) : 1.0f;
  const bool qfast = quot_divisor_ok(sx);
  const float rsx = __frcp_rn(sx);
  int parity = 0;
  // x (and r) of a row, loaded by this thread; the next row's are issued
  // before the current row is reduced, so two rows per CTA are in flight.
  uint4 xv[NV], rv[NV], xn[NV], rn_[NV];
  auto load_row = [&](int row, uint4 (&xa)[NV], uint4 (&ra)[NV]) {
    const uint4* xr = reinterpret_cast<const uint4*>(A.x + (long long)row * A.ldx);
    const uint4* rr =
        A.r != nullptr ? reinterpret_cast<const uint4*>(A.r + (long long)row * A.ldr) : nullptr;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = tid + i * NORM_THREADS;
      if (v < vpr) {
        xa[i] = __ldcs(xr + v);
        if (A.r != nullptr) ra[i] = __ldcs(rr + v);
      }
    }
  };
  if ((int)blockIdx.x < A.M) load_row((int)blockIdx.x, xv, rv);
  for (int row = blockIdx.x; row < A.M; row += gridDim.x, parity ^= 1) {
    if (row + (int)gridDim.x < A.M) load_row(row + (int)gridDim.x, xn, rn_);
    if (A.r != nullptr) {
      // bf16 + bf16 -> bf16: the exact sum rounded once (see packed math)
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        uint32_t* a = reinterpret_cast<uint32_t*>(&xv[i]);
        const uint32_t* b = reinterpret_cast<const uint32_t*>(&rv[i]);
#pragma unroll
        for (int k = 0; k < 4; ++k) a[k] = as_u32(__hadd2(as_bf162(a[k]), as_bf162(b[k])));
      }
    }
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (tid + i * NORM_THREADS >= vpr) continue;
      const uint32_t* a = reinterpret_cast<const uint32_t*>(&xv[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = bf2f(a[k]);
        acc = fmaf(f.x, f.x, acc);  // squares of bf16 values are exact in fp32
        acc = fmaf(f.y, f.y, acc);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) red[parity][warp] = acc;
    __syncthreads();  // red[parity] complete; red[parity ^ 1] is free for the next row
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < NORM_THREADS / 32; ++w) tot += red[parity][w];
    float n = bf16r(__fsqrt_rn(tot));
    n = bf16r(n * A.inv_sqrt_h);
    n = bf16r(n + A.eps);
    const bool nfast = quot_divisor_ok(n);
    const float rn = __frcp_rn(n);

#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = tid + i * NORM_THREADS;
      if (v >= vpr) continue;
      if (A.s != nullptr)
        __stcs(reinterpret_cast<uint4*>(A.s + (long long)row * A.lds) + v, xv[i]);
      const uint32_t* a = reinterpret_cast<const uint32_t*>(&xv[i]);
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(A.w) + v);  // L1-resident
      const uint32_t* wk = reinterpret_cast<const uint32_t*>(&wv);
      float y[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = bf2f(a[k]), g = bf2f(wk[k]);
        y[2 * k] = bf16r(g.x * quot_bf16(f.x, n, rn, nfast));
        y[2 * k + 1] = bf16r(g.y * quot_bf16(f.y, n, rn, nfast));
      }
      if (A.y != nullptr) {
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) ow[k] = as_u32(pack2_rn(make_float2(y[2 * k], y[2 * k + 1])));
        __stcs(reinterpret_cast<uint4*>(A.y + (long long)row * A.ldy) + v, o);
      }
      if (A.q != nullptr) {
        __nv_fp8x2_storage_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = quot_e4m3x2(y[2 * k], y[2 * k + 1], sx, rsx, qfast);
        reinterpret_cast<uint2*>(A.q + (long long)row * A.ldq)[v] =
            *reinterpret_cast<const uint2*>(o);
      }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      xv[i] = xn[i];
      rv[i] = rn_[i];
    }
  }
}

// One resident wave: blocks = SMs x the blocks of this variant an SM holds.
template <int NV>
static int launch_norm(const NormArgs& A, cudaStream_t st) {
  static const int per_sm = [] {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, rms_norm_kernel<NV>, NORM_THREADS, 0) !=
            cudaSuccess || n < 1)
      n = 4;
    return n;
  }();
  const int wave = num_sms() * per_sm;
  launch_kernel(rms_norm_kernel<NV>, dim3(A.M < wave ? A.M : wave), dim3(NORM_THREADS), 0, st, 0u,
                A);
  return check_launch("rms_norm_kernel");
}

int rms_norm_launch(const NormArgs& A, cudaStream_t st) {
  if (A.M <= 0) return HYENA_OK;
  HB_REQUIRE(A.x && A.w, "rms_norm: null x or weight");
  HB_REQUIRE(A.H > 0 && A.H % 8 == 0 && A.H <= 16 * 8 * NORM_THREADS,
             "rms_norm: H must be a positive multiple of 8, at most 16384");
  HB_REQUIRE(A.y || A.q || A.s, "rms_norm: no output requested");
  HB_REQUIRE(!A.q || A.sx, "rms_norm: q requested without an input scale");
  HB_REQUIRE(aligned16(A.x) && A.ldx % 8 == 0 && aligned16(A.w), "rms_norm: x / weight misaligned");
  HB_REQUIRE(!A.r || (aligned16(A.r) && A.ldr % 8 == 0), "rms_norm: residual misaligned");
  HB_REQUIRE(!A.s || (aligned16(A.s) && A.lds % 8 == 0), "rms_norm: s_out misaligned");
  HB_REQUIRE(!A.y || (aligned16(A.y) && A.ldy % 8 == 0), "rms_norm: y misaligned");
  HB_REQUIRE(!A.q || ((reinterpret_cast<uintptr_t>(A.q) & 7u) == 0 && A.ldq % 8 == 0),
             "rms_norm: q misaligned");
  const int vpr = A.H / 8;
  const int nv = (vpr + NORM_THREADS - 1) / NORM_THREADS;
  if (nv <= 1) return launch_norm<1>(A, st);
  if (nv <= 2) return launch_norm<2>(A, st);
  if (nv <= 4) return launch_norm<4>(A, st);
  if (nv <= 8) return launch_norm<8>(A, st);
  return launch_norm<16>(A, st);
}

}  // namespace hb
