// Shared helpers for the Hyena-mixer kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "hyena_b200.h"

namespace hb {

typedef __nv_bfloat16 bf16;

// ---------------------------------------------------------------- host errors
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_launch(const char* what);

#define HB_REQUIRE(cond, msg)                                    \
  do {                                                           \
    if (!(cond)) return ::hb::fail(HYENA_ERR_INVALID, (msg));    \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- device math
// Round to bf16 and back: the value a torch op with a bf16 output stores.
__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float ldbf(const bf16* p) { return __bfloat162float(*p); }

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
