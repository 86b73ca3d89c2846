// Shared helpers for the Hyena-mixer kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "hyena_b200.h"

namespace hb {

typedef __nv_bfloat16 bf16;

// ---------------------------------------------------------------- host errors
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_launch(const char* what);

// Arguments of the decoder-layer norm (hyena_rms_norm).
struct NormArgs {
  const bf16* x;
  int64_t ldx;
  const bf16* r;  // residual or null
  int64_t ldr;
  const bf16* w;  // (H)
  bf16* s;        // x + r, or null
  int64_t lds;
  bf16* y;        // normed output, or null
  int64_t ldy;
  uint8_t* q;     // e4m3 output, or null
  int64_t ldq;
  const float* sx;  // e4m3 input scale (q only)
  int M, H;
  float inv_sqrt_h, eps;
};

int rms_norm_launch(const NormArgs& A, cudaStream_t st);

#define HB_REQUIRE(cond, msg)                                    \
  do {                                                           \
    if (!(cond)) return ::hb::fail(HYENA_ERR_INVALID, (msg));    \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- launches
// Every kernel of the library is launched with programmatic dependent launch,
// so that it can be scheduled while the previous kernel in the stream drains.
// In every thread a kernel calls pdl_wait() (returns once the previous kernel
// has completed and its writes are visible) before its first load or store of
// global memory that other kernels write or read, and only after that wait
// lets its own successor launch (pdl_trigger: the successor's CTAs may start
// once every CTA of this grid has triggered or exited).  Before the wait go
// shared-memory / TMEM set-up and tensor-map or L2 prefetches only.
//
// Because no kernel triggers before its wait returns, at most two kernels of a
// stream are resident at a time: the running one and its successor doing its
// set-up.  Triggering at entry instead let whole chains of successors become
// resident early and wait; the speculative verify step (18 launches) took
// 0.529 ms that way against 0.500 ms now, ordinary decode 0.2282 against
// 0.2274 ms.  (The SM-pair GEMM is launched without the programmatic
// attribute, so it starts after its predecessor completes; it triggers at
// entry.)  Without a programmatic predecessor pdl_wait() returns at once.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_entry() {
  pdl_wait();
  pdl_trigger();
}

// SMs of the current device (148 on B200).
inline int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    sms = (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
              ? n : 148;
  }
  return sms;
}

// cudaFuncSetAttribute(Kern, MaxDynamicSharedMemorySize, bytes) once per
// device (a function attribute belongs to the device's context).
constexpr int HB_MAX_DEVICES = 64;
template <auto Kern>
inline bool smem_attr(int bytes) {
  static std::atomic<int> done[HB_MAX_DEVICES];  // bytes set per device (0: none)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= HB_MAX_DEVICES) return false;
  if (done[dev].load(std::memory_order_relaxed) == bytes) return true;
  if (cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return false;
  done[dev].store(bytes, std::memory_order_relaxed);
  return true;
}

// Process-wide switch for the programmatic-serialisation attribute (on by
// default; hyena_set_launch_chaining).
bool launch_chaining();

// cudaLaunchKernelEx with the programmatic-serialisation attribute (and a
// 1-D cluster of `cluster_x` CTAs when cluster_x > 0).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t st, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  unsigned n = 0;
  if (launch_chaining()) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 0) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = cluster_x;
    at[n].val.clusterDim.y = 1;
    at[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

// ---------------------------------------------------------------- device math
// Round to bf16 and back: the value a torch op with a bf16 output stores.
__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float ldbf(const bf16* p) { return __bfloat162float(*p); }

// ---------------------------------------------------------------- cp.async
// 16-byte global -> shared copies (L2 only), grouped and waited on per group.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- quotients
// A divide by a per-row or per-tensor divisor b whose fp32 quotient is then
// rounded to a narrow type (bf16 or e4m3), with the result of the correctly
// rounded __fdiv_rn but mostly at the cost of a multiply.  rb = __frcp_rn(b);
// for b in [2^-125, 2^125] and a normal fp32 product p = fl(a * rb), p differs
// from a / b by at most 2^-23 |a / b| (two roundings of relative error 2^-24),
// so it lies within 3 ulps of fl(a / b) in its binade, within 6 encodings
// across a binade edge.  Rounding to the narrow type is monotonic and changes
// value only at its ties, which are fp32 encodings with fixed low bits (bf16:
// low 16 bits 0x8000; normal e4m3, |p| >= 2^-6: low 20 bits 0x80000); when no
// tie lies within 8 encodings of p, fl(a / b) rounds to the same value as p.
// Otherwise (p near a tie, subnormal, zero, or an e4m3 subnormal) the quotient
// is recomputed with __fdiv_rn.  e4m3 saturates at 448, so p beyond the normal
// range (even inf) needs no check.
__device__ __forceinline__ bool quot_divisor_ok(float b) {
  const float m = fabsf(b);
  return m >= 0x1p-125f && m <= 0x1p125f;
}
// No bf16 tie within 8 encodings of p, and p a normal number.
__device__ __forceinline__ bool quot_bf16_clear(uint32_t u) {
  return ((u + 0x8008u) & 0xFFFFu) > 16u && ((u & 0x7F800000u) - 0x00800000u) < 0x7F000000u;
}
// No e4m3 tie within 8 encodings of p, and |p| >= 2^-6 (e4m3 normal or beyond).
__device__ __forceinline__ bool quot_e4m3_clear(uint32_t u) {
  return ((u + 0x80008u) & 0xFFFFFu) > 16u && (u & 0x7FFFFFFFu) >= 0x3C800000u;
}
// a / b rounded to bf16 (returned as fp32).
__device__ __forceinline__ float quot_bf16(float a, float b, float rb, bool fast) {
  const float p = a * rb;
  if (fast && quot_bf16_clear(__float_as_uint(p))) return bf16r(p);
  return bf16r(__fdiv_rn(a, b));
}
// (a0, a1) / b as a saturating e4m3 pair: clamp to +-448 then round to nearest
// even (NaN stays NaN), the quantisation of fp8_emul.quantize_input
// (fp8_emul.py:76-78).
__device__ __forceinline__ __nv_fp8x2_storage_t e4m3x2(float x0, float x1) {
  return __nv_cvt_float2_to_fp8x2(make_float2(x0, x1), __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ __nv_fp8x2_storage_t quot_e4m3x2(float a0, float a1, float b, float rb,
                                                             bool fast) {
  const float p0 = a0 * rb, p1 = a1 * rb;
  if (fast && quot_e4m3_clear(__float_as_uint(p0)) && quot_e4m3_clear(__float_as_uint(p1)))
    return e4m3x2(p0, p1);
  return e4m3x2(__fdiv_rn(a0, b), __fdiv_rn(a1, b));
}

// Multiply and add with separate roundings (no FMA contraction): the order of
// an eager torch recurrence s = s * p + x.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

__device__ __forceinline__ void flag_error(int32_t* flags, int bit) {
  if (flags) atomicOr(flags, bit);
}

// vLLM's K=3 short-filter step: fp32 accumulator over three products each
// rounded to bf16, oldest tap first, result rounded to bf16
// (vLLM causal_conv1d kernels; restated in evo2_flash/triton_decode.py:43-53).
__device__ __forceinline__ float short_tap(float c0, float c1, float x, float w0, float w1,
                                           float w2) {
  float acc = 0.0f;
  acc = add_rn(acc, bf16r(c0 * w0));
  acc = add_rn(acc, bf16r(c1 * w1));
  acc = add_rn(acc, bf16r(x * w2));
  return bf16r(acc);
}

// Readout y = sum_s R_s * s_s over 16 modes with the halving tree
// p[s] += p[s+8]; += p[s+4]; += p[s+2]; += p[s+1]; take p[0]
// (evo2_flash/triton_decode.py:89-93, triton_verifier.py:115-119).
__device__ __forceinline__ float modal_readout16(const float* s, const float* r) {
  float p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) p[i] = mul_rn(s[i], r[i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = add_rn(p[i], p[i + 8]);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = add_rn(p[i], p[i + 4]);
#pragma unroll
  for (int i = 0; i < 2; ++i) p[i] = add_rn(p[i], p[i + 2]);
  return add_rn(p[0], p[1]);
}

// ---------------------------------------------------------------- packed math
// bf16x2 / f32x2 helpers.  A bf16x2 product is the correctly rounded bf16 of
// the exact product (the rounding a torch bf16 multiply performs), and a bf16x2
// sum of two bf16 values equals torch's fp32-add-then-round (the exact sum of
// two bf16 numbers either fits fp32 or the smaller term is below half an ulp).
typedef __nv_bfloat162 bf162;

__device__ __forceinline__ bf162 as_bf162(uint32_t v) { return *reinterpret_cast<bf162*>(&v); }
__device__ __forceinline__ uint32_t as_u32(bf162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// (lo, hi) of a bf16x2 as fp32
__device__ __forceinline__ float2 unpack2(bf162 v) { return __bfloat1622float2(v); }

__device__ __forceinline__ bf162 pack2_rn(float2 v) { return __floats2bfloat162_rn(v.x, v.y); }

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long ra, rb, rc;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rc) : "l"(ra), "l"(rb));
  float2 c;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(c.x), "=f"(c.y) : "l"(rc));
  return c;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  unsigned long long ra, rb, rc;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(rc) : "l"(ra), "l"(rb));
  float2 c;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(c.x), "=f"(c.y) : "l"(rc));
  return c;
}

// modal_readout16 on mode pairs (s2[i] = modes 2i, 2i+1): the same halving
// tree, two modes per instruction.
__device__ __forceinline__ float modal_readout16_x2(const float2* s2, const float2* r2) {
  float2 p[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = fmul2(s2[i], r2[i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = fadd2(p[i], p[i + 4]);
#pragma unroll
  for (int i = 0; i < 2; ++i) p[i] = fadd2(p[i], p[i + 2]);
  p[0] = fadd2(p[0], p[1]);
  return add_rn(p[0].x, p[0].y);
}

// c + a * b, elementwise on two fp32 lanes, one rounding each (fmaf per lane).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long ra, rb, rc, rd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rc) : "f"(c.x), "f"(c.y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  float2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(rd));
  return d;
}

// Two fp32 lanes held in one 64-bit register (lo = first element).  Keeping
// packed values in this type end to end lets fma/mul/add.f32x2 run without
// register-pair shuffles.
typedef unsigned long long f2;

__device__ __forceinline__ f2 f2_make(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_split(f2 v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ f2 f2_fma(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 f2_add(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// bf16x2 word -> two fp32 lanes (exact)
__device__ __forceinline__ f2 f2_from_bf162(bf162 v) {
  const uint32_t w = as_u32(v);
  return (f2)(w << 16) | ((f2)(w & 0xffff0000u) << 32);
}
// two fp32 lanes -> bf16x2, round to nearest even
__device__ __forceinline__ bf162 bf162_from_f2(f2 v) {
  const float2 x = f2_split(v);
  return __floats2bfloat162_rn(x.x, x.y);
}

// short_tap on a channel pair: products rounded to bf16 (bf16x2 multiply),
// summed oldest first in fp32 from a +0 accumulator, result rounded to bf16.
// The sums use the mixed-precision add (a bf16 operand added to an fp32 one,
// one fp32 rounding), so the bf16 products need no unpacking into fp32.
__device__ __forceinline__ bf162 short_tap2(bf162 c0, bf162 c1, bf162 x, bf162 w0, bf162 w1,
                                            bf162 w2) {
  const uint32_t p0 = as_u32(__hmul2(c0, w0));
  const uint32_t p1 = as_u32(__hmul2(c1, w1));
  const uint32_t p2 = as_u32(__hmul2(x, w2));
  float lo, hi;
  asm("{\n\t.reg .b16 a0, a1, b0, b1, e0, e1;\n\t"
      "mov.b32 {a0, a1}, %2;\n\tmov.b32 {b0, b1}, %3;\n\tmov.b32 {e0, e1}, %4;\n\t"
      "add.rn.f32.bf16 %0, a0, 0f00000000;\n\tadd.rn.f32.bf16 %1, a1, 0f00000000;\n\t"
      "add.rn.f32.bf16 %0, b0, %0;\n\tadd.rn.f32.bf16 %1, b1, %1;\n\t"
      "add.rn.f32.bf16 %0, e0, %0;\n\tadd.rn.f32.bf16 %1, e1, %1;\n\t}"
      : "=&f"(lo), "=&f"(hi)
      : "r"(p0), "r"(p1), "r"(p2));
  return __floats2bfloat162_rn(lo, hi);
}

// Largest j with qsl[j] <= row, for a non-decreasing qsl[0..n].
__device__ __forceinline__ int find_segment(const int32_t* qsl, int n, int row) {
  int lo = 0, hi = n;  // invariant: answer in [lo, hi)
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (__ldg(qsl + mid) <= row) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace hb
