// Hyena-LI (HCL) prefill for sm_100a: the order-16 diagonal modal SSM
//     s_t = p (.) s_{t-1} + u_t,   y_t = sum_s R_s s_{t,s},   p = exp(log_poles)
// over packed varlen segments, fused with the K=3 short filter, the x1*v gate
// and the (y + D*u) * x2 output gate.
//
// The reference computes the same map as an FFT convolution with the
// materialised modal filter h[t] = sum_s R_s p_s^t plus a closed-form final
// state and the s_prev continuation terms (mixers.py:144-210, 1378-1397;
// triton_hcl.py; triton_prefill.py:351-387).  Unrolling the recurrence gives
// exactly those terms, so here the scan itself is the algorithm: no filter, no
// FFT, O(16) work per element and the final state falls out as the carry.
//
// Parallel form (time-chunked scan, C rows per chunk, chunks never straddle a
// segment boundary):
//   plan      chunk_base[j] = number of chunks before segment j       (1 CTA)
//   aggregate A_c = sum_{tau in chunk} p^(C-1-tau) u_tau  for every non-final chunk
//   carry     S_in[c+1] = p^C (.) S_in[c] + A_c, S_in[first] = cached state or 0
//   output    rerun the recurrence from S_in over the chunk, write g, and the
//             final chunk of each segment stores its end state into S2.
// Every launch is order-independent across CTAs: no inter-CTA waits.
#include "common.cuh"

namespace hb {

constexpr int HCL_C = 256;       // rows per chunk
constexpr int HCL_CG = 128;      // channels per CTA (one thread per channel)
constexpr int HCL_TILE = 32;     // rows staged in shared memory at a time
constexpr int HCL_S = 16;        // modal order

struct HclWorkspace {
  int32_t* chunk_base;  // (nseg + 1)
  float* states;        // (max_chunks, H, 16)
};

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

size_t hcl_workspace_size(int H, int T, int nseg) {
  const size_t max_chunks = (size_t)(T + HCL_C - 1) / HCL_C + (size_t)nseg;
  return align_up(sizeof(int32_t) * (size_t)(nseg + 1), 256) +
         sizeof(float) * max_chunks * (size_t)H * HCL_S;
}

static HclWorkspace carve(void* ws, int nseg) {
  HclWorkspace w;
  w.chunk_base = static_cast<int32_t*>(ws);
  w.states = reinterpret_cast<float*>(static_cast<char*>(ws) +
                                      align_up(sizeof(int32_t) * (size_t)(nseg + 1), 256));
  return w;
}

__global__ void hcl_plan_kernel(const int32_t* qsl, int nseg, int32_t* chunk_base) {
  if (threadIdx.x != 0) return;
  int acc = 0;
  for (int j = 0; j < nseg; ++j) {
    chunk_base[j] = acc;
    const int L = __ldg(qsl + j + 1) - __ldg(qsl + j);
    acc += L > 0 ? (L + HCL_C - 1) / HCL_C : 0;
  }
  chunk_base[nseg] = acc;
}

struct ChunkCtx {
  int seg, k, nch;  // segment, chunk within segment, chunks of the segment
  int a, e;         // segment rows
  int row0, row1;   // chunk rows
  long long blk;
  bool init;
};

// Returns false when this CTA has no chunk.
__device__ __forceinline__ bool chunk_ctx(const hyena_prefill_args& A, const int32_t* cb,
                                          int ci, ChunkCtx& c) {
  const int nseg = A.num_segments;
  if (ci >= __ldg(cb + nseg)) return false;
  const int j = find_segment(cb, nseg, ci);  // last j with cb[j] <= ci (skips empty segments)
  // Segments with zero chunks share their base with the next one; find_segment
  // returns the last j with cb[j] <= ci, which is the non-empty owner.
  c.seg = j;
  c.k = ci - __ldg(cb + j);
  c.nch = __ldg(cb + j + 1) - __ldg(cb + j);
  c.a = __ldg(A.query_start_loc + j);
  c.e = __ldg(A.query_start_loc + j + 1);
  c.row0 = c.a + c.k * HCL_C;
  c.row1 = min(c.e, c.row0 + HCL_C);
  c.blk = __ldg(A.state_indices + (long long)j * A.state_indices_stride);
  c.init = A.has_initial_state != nullptr && __ldg(A.has_initial_state + j) != 0;
  return true;
}

// Stages z rows [t0, t0+n) x (3*HCL_CG) columns into shared memory.
__device__ __forceinline__ void stage_rows(const hyena_prefill_args& A, bf16 (*zt)[3 * HCL_CG],
                                           int t0, int n, int c0) {
  const bf16* z = static_cast<const bf16*>(A.z);
  constexpr int VPR = 3 * HCL_CG * 2 / 16;
  for (int i = threadIdx.x; i < n * VPR; i += HCL_CG) {
    const int row = i / VPR, v = i % VPR;
    *(reinterpret_cast<uint4*>(&zt[row][0]) + v) =
        __ldg(reinterpret_cast<const uint4*>(z + (long long)(t0 + row) * A.ldz + 3 * c0) + v);
  }
}

// z at row t < a (left context of a segment) for column col: cached S0 or zero.
__device__ __forceinline__ float z_before(const hyena_prefill_args& A, const ChunkCtx& c,
                                          long long t, int col) {
  if (!c.init) return 0.0f;
  const long long back = c.a - t;  // 1 = newest cached input, in column 1
  if (back > 2) return 0.0f;
  const bf16* s0 = static_cast<const bf16*>(A.conv_state.data);
  return ldbf(s0 + c.blk * A.conv_state.block_stride + (2 - back) * A.conv_state.col_stride +
              (long long)col * A.conv_state.dim_stride);
}

__device__ __forceinline__ float z_global(const hyena_prefill_args& A, const ChunkCtx& c,
                                          long long t, int col) {
  if (t >= c.a) return ldbf(static_cast<const bf16*>(A.z) + t * A.ldz + col);
  return z_before(A, c, t, col);
}

// Walks the chunk's rows, calling fn(row, x2, u) in order for this thread's channel.
template <bool NEED_X2, typename F>
__device__ __forceinline__ void walk_chunk(const hyena_prefill_args& A,
                                           const hyena_layer_params& P, const ChunkCtx& c,
                                           int c0, bf16 (*zt)[3 * HCL_CG], F&& fn) {
  const int tid = threadIdx.x;
  const int h = c0 + tid;
  const bf16* sw = static_cast<const bf16*>(P.short_w);
  float w[3][3];
#pragma unroll
  for (int q = 0; q < 3; ++q)
#pragma unroll
    for (int t = 0; t < 3; ++t) w[q][t] = ldbf(sw + (3 * h + q) * 3 + t);
  // z history (rows row0-2, row0-1) of the three columns
  float hm2[3], hm1[3];
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    hm2[q] = z_global(A, c, (long long)c.row0 - 2, 3 * h + q);
    hm1[q] = z_global(A, c, (long long)c.row0 - 1, 3 * h + q);
  }
  for (int t0 = c.row0; t0 < c.row1; t0 += HCL_TILE) {
    const int n = min(HCL_TILE, c.row1 - t0);
    __syncthreads();
    stage_rows(A, zt, t0, n, c0);
    __syncthreads();
    for (int row = 0; row < n; ++row) {
      float o[3];
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        if (!NEED_X2 && q == 0) { o[0] = 0.0f; continue; }
        const float x0 = __bfloat162float(zt[row][3 * tid + q]);
        o[q] = short_tap(hm2[q], hm1[q], x0, w[q][0], w[q][1], w[q][2]);
        hm2[q] = hm1[q];
        hm1[q] = x0;
      }
      fn(t0 + row, o[0], bf16r(o[1] * o[2]));
    }
  }
}

__device__ __forceinline__ void load_poles(const hyena_layer_params& P, int h, float* p) {
#pragma unroll
  for (int s = 0; s < HCL_S; ++s) p[s] = expf(P.log_poles[(long long)h * P.lp_stride_h + s * P.lp_stride_s]);
}

__global__ void __launch_bounds__(HCL_CG)
hcl_aggregate_kernel(const hyena_layer_params P, const hyena_prefill_args A, HclWorkspace W) {
  __shared__ __align__(16) bf16 zt[HCL_TILE][3 * HCL_CG];
  ChunkCtx c;
  if (!chunk_ctx(A, W.chunk_base, blockIdx.x, c)) return;
  if (c.k == c.nch - 1) return;  // the final chunk's aggregate is never needed
  const int c0 = blockIdx.y * HCL_CG;
  const int h = c0 + threadIdx.x;
  if (c.init && (c.blk < 0 || c.blk >= A.conv_state.num_blocks)) c.init = false;
  float p[HCL_S], acc[HCL_S];
  load_poles(P, h, p);
#pragma unroll
  for (int s = 0; s < HCL_S; ++s) acc[s] = 0.0f;
  walk_chunk<false>(A, P, c, c0, zt, [&](int, float, float u) {
#pragma unroll
    for (int s = 0; s < HCL_S; ++s) acc[s] = add_rn(mul_rn(acc[s], p[s]), u);
  });
  float4* dst = reinterpret_cast<float4*>(W.states + ((long long)blockIdx.x * P.H + h) * HCL_S);
#pragma unroll
  for (int s = 0; s < HCL_S / 4; ++s)
    dst[s] = make_float4(acc[4 * s], acc[4 * s + 1], acc[4 * s + 2], acc[4 * s + 3]);
}

// One thread per (segment, channel): S_in for every chunk, written over the
// chunk's aggregate.
__global__ void __launch_bounds__(128)
hcl_carry_kernel(const hyena_layer_params P, const hyena_prefill_args A, HclWorkspace W) {
  const int j = blockIdx.x;
  const int h = blockIdx.y * 128 + threadIdx.x;
  if (h >= P.H) return;
  const int base = __ldg(W.chunk_base + j);
  const int nch = __ldg(W.chunk_base + j + 1) - base;
  if (nch <= 0) return;
  const long long blk = __ldg(A.state_indices + (long long)j * A.state_indices_stride);
  bool init = A.has_initial_state != nullptr && __ldg(A.has_initial_state + j) != 0;
  if (init && (blk < 0 || blk >= A.inner_state.num_blocks)) {
    flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    init = false;
  }
  float S[HCL_S], pc[HCL_S];
  const float* s2 = static_cast<const float*>(A.inner_state.data);
#pragma unroll
  for (int s = 0; s < HCL_S; ++s) {
    S[s] = init ? s2[blk * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
                     (long long)s * A.inner_state.col_stride]
                : 0.0f;
    pc[s] = expf(P.log_poles[(long long)h * P.lp_stride_h + s * P.lp_stride_s] * (float)HCL_C);
  }
  for (int k = 0; k < nch; ++k) {
    float4* slot = reinterpret_cast<float4*>(W.states + ((long long)(base + k) * P.H + h) * HCL_S);
    float a[HCL_S];
    if (k < nch - 1) {
#pragma unroll
      for (int s = 0; s < HCL_S / 4; ++s) {
        const float4 v = slot[s];
        a[4 * s] = v.x; a[4 * s + 1] = v.y; a[4 * s + 2] = v.z; a[4 * s + 3] = v.w;
      }
    }
#pragma unroll
    for (int s = 0; s < HCL_S / 4; ++s)
      slot[s] = make_float4(S[4 * s], S[4 * s + 1], S[4 * s + 2], S[4 * s + 3]);
    if (k < nch - 1) {
#pragma unroll
      for (int s = 0; s < HCL_S; ++s) S[s] = add_rn(mul_rn(pc[s], S[s]), a[s]);
    }
  }
}

__global__ void __launch_bounds__(HCL_CG)
hcl_output_kernel(const hyena_layer_params P, const hyena_prefill_args A, HclWorkspace W) {
  __shared__ __align__(16) bf16 zt[HCL_TILE][3 * HCL_CG];
  ChunkCtx c;
  if (!chunk_ctx(A, W.chunk_base, blockIdx.x, c)) return;
  const int c0 = blockIdx.y * HCL_CG;
  const int h = c0 + threadIdx.x;
  const bool blk_ok = c.blk >= 0 && c.blk < A.inner_state.num_blocks &&
                      c.blk < A.conv_state.num_blocks;
  if (c.init && !blk_ok) c.init = false;
  float p[HCL_S], r[HCL_S], s[HCL_S];
  load_poles(P, h, p);
#pragma unroll
  for (int q = 0; q < HCL_S; ++q) r[q] = P.residues[(long long)h * P.res_stride_h + q * P.res_stride_s];
  {
    const float4* src =
        reinterpret_cast<const float4*>(W.states + ((long long)blockIdx.x * P.H + h) * HCL_S);
#pragma unroll
    for (int q = 0; q < HCL_S / 4; ++q) {
      const float4 v = src[q];
      s[4 * q] = v.x; s[4 * q + 1] = v.y; s[4 * q + 2] = v.z; s[4 * q + 3] = v.w;
    }
  }
  const bf16* Dg = static_cast<const bf16*>(P.D);
  const float d = Dg ? ldbf(Dg + h) : 0.0f;
  bf16* out = static_cast<bf16*>(A.out);
  walk_chunk<true>(A, P, c, c0, zt, [&](int row, float x2, float u) {
#pragma unroll
    for (int q = 0; q < HCL_S; ++q) s[q] = add_rn(mul_rn(s[q], p[q]), u);
    float y = bf16r(modal_readout16(s, r));
    if (Dg) y = bf16r(y + bf16r(u * d));
    out[(long long)row * A.ldo + h] = __float2bfloat16_rn(bf16r(y * x2));
  });
  if (c.k == c.nch - 1) {
    if (!blk_ok) {
      if (threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
      return;
    }
    float* s2 = static_cast<float*>(A.inner_state.data);
#pragma unroll
    for (int q = 0; q < HCL_S; ++q)
      s2[c.blk * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
         (long long)q * A.inner_state.col_stride] = s[q];
  }
}

int conv_state_update_launch(const hyena_layer_params& P, const hyena_prefill_args& A,
                             cudaStream_t st);

int hcl_prefill_launch(const hyena_layer_params& P, const hyena_prefill_args& A, void* ws,
                       size_t ws_bytes, cudaStream_t st) {
  if (P.K != HCL_S) return fail(HYENA_ERR_UNSUPPORTED, "HCL prefill supports modal order 16");
  if (P.H % HCL_CG) return fail(HYENA_ERR_INVALID, "HCL prefill needs H % 128 == 0");
  const size_t need = hcl_workspace_size(P.H, A.T, A.num_segments);
  if (ws == nullptr || ws_bytes < need)
    return fail(HYENA_ERR_INVALID, "HCL prefill workspace too small");
  if (!aligned16(ws)) return fail(HYENA_ERR_INVALID, "HCL workspace must be 16-byte aligned");
  HclWorkspace W = carve(ws, A.num_segments);
  const int max_chunks = (A.T + HCL_C - 1) / HCL_C + A.num_segments;
  const int groups = P.H / HCL_CG;
  hcl_plan_kernel<<<1, 32, 0, st>>>(A.query_start_loc, A.num_segments, W.chunk_base);
  int rc = check_launch("hcl_plan_kernel");
  if (rc) return rc;
  hcl_aggregate_kernel<<<dim3(max_chunks, groups), HCL_CG, 0, st>>>(P, A, W);
  if ((rc = check_launch("hcl_aggregate_kernel"))) return rc;
  hcl_carry_kernel<<<dim3(A.num_segments, (P.H + 127) / 128), 128, 0, st>>>(P, A, W);
  if ((rc = check_launch("hcl_carry_kernel"))) return rc;
  hcl_output_kernel<<<dim3(max_chunks, groups), HCL_CG, 0, st>>>(P, A, W);
  if ((rc = check_launch("hcl_output_kernel"))) return rc;
  return conv_state_update_launch(P, A, st);
}

}  // namespace hb
