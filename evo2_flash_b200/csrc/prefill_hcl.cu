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
constexpr int HCL_TILE = 16;     // rows staged in shared memory at a time
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
  pdl_entry();
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

struct HclTile {
  uint32_t zt[2][HCL_TILE][3 * HCL_CG / 2];  // z rows, raw bf16x2 words (double-buffered)
  uint32_t zh[2][3 * HCL_CG / 2];            // the two z rows before the tile
  bf162 ug[HCL_TILE][HCL_CG / 2];         // u = bf16(x1*v), channel pairs
  bf162 x2g[HCL_TILE][HCL_CG / 2];
};

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

__device__ __forceinline__ void split_triples_hcl(uint32_t w0, uint32_t w1, uint32_t w2,
                                                  bf162& x2, bf162& x1, bf162& v) {
  x2 = as_bf162(__byte_perm(w0, w1, 0x7610));
  x1 = as_bf162(__byte_perm(w0, w2, 0x5432));
  v = as_bf162(__byte_perm(w1, w2, 0x7610));
}

// Walks the chunk's rows in tiles: all threads stage the z rows and run the K=3
// filter + gate on channel pairs (bf16x2), then fn(row, x2, u) is called in row
// order with this thread's channel.  NEED_X2 = false (the aggregate pass, which
// uses u only) skips the x2 column's filter; fn then gets x2 = 0.
template <bool NEED_X2, typename F>
__device__ __forceinline__ void walk_chunk(const hyena_prefill_args& A,
                                           const hyena_layer_params& P, const ChunkCtx& c,
                                           int c0, HclTile& S, F&& fn) {
  const int tid = threadIdx.x;
  constexpr int PAIRS = HCL_CG / 2;
  constexpr int WORDS = 3 * HCL_CG / 2;
  const int pp = tid % PAIRS;   // gate: channel pair
  const int half = tid / PAIRS; // gate: rows [16 half, 16 half + 16) of the tile
  const bf16* sw = static_cast<const bf16*>(P.short_w);
  bf162 w[3][3];
  {
    const long long h = c0 + 2 * pp;
#pragma unroll
    for (int col = 0; col < 3; ++col)
#pragma unroll
      for (int t = 0; t < 3; ++t)
        w[col][t] = __halves2bfloat162(sw[(3 * h + col) * 3 + t], sw[(3 * (h + 1) + col) * 3 + t]);
  }
  for (int i = tid; i < 2 * WORDS; i += HCL_CG) {
    const int q = i / WORDS, wd = i % WORDS;
    const long long t = (long long)c.row0 - 2 + q;
    const uint32_t lo = (uint32_t)__bfloat16_as_ushort(
        __float2bfloat16_rn(z_global(A, c, t, 3 * c0 + 2 * wd)));
    const uint32_t hi = (uint32_t)__bfloat16_as_ushort(
        __float2bfloat16_rn(z_global(A, c, t, 3 * c0 + 2 * wd + 1)));
    S.zh[q][wd] = lo | (hi << 16);
  }
  const bf16* z = static_cast<const bf16*>(A.z);
  constexpr int VPR = WORDS * 4 / 16;  // 16-byte vectors per z row of the CTA
  // Tile k's z rows into buffer k & 1 with cp.async; one group per call.
  auto issue = [&](int t0) {
    if (t0 < c.row1) {
      const int n = min(HCL_TILE, c.row1 - t0);
      uint32_t(*dst)[WORDS] = S.zt[((t0 - c.row0) / HCL_TILE) & 1];
      for (int i = tid; i < n * VPR; i += HCL_CG) {
        const int row = i / VPR, v = i % VPR;
        cp_async16(reinterpret_cast<uint4*>(&dst[row][0]) + v,
                   reinterpret_cast<const uint4*>(z + (long long)(t0 + row) * A.ldz + 3 * c0) + v);
      }
    }
    cp_async_commit();
  };
  issue(c.row0);
  for (int t0 = c.row0; t0 < c.row1; t0 += HCL_TILE) {
    const int n = min(HCL_TILE, c.row1 - t0);
    issue(t0 + HCL_TILE);  // the next tile loads while this one is processed
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t(*zt)[WORDS] = S.zt[((t0 - c.row0) / HCL_TILE) & 1];
    {
      const int g0 = half * (HCL_TILE / 2);
      bf162 h2[3], h1[3];
      const uint32_t* a = g0 >= 2 ? &zt[g0 - 2][3 * pp] : &S.zh[g0][3 * pp];
      const uint32_t* b = g0 >= 1 ? &zt[g0 - 1][3 * pp] : &S.zh[1][3 * pp];
      split_triples_hcl(a[0], a[1], a[2], h2[0], h2[1], h2[2]);
      split_triples_hcl(b[0], b[1], b[2], h1[0], h1[1], h1[2]);
#pragma unroll 4
      for (int i = 0; i < HCL_TILE / 2; ++i) {
        const int row = g0 + i;
        if (row < n) {
          bf162 cur[3], o[3];
          split_triples_hcl(zt[row][3 * pp], zt[row][3 * pp + 1], zt[row][3 * pp + 2],
                            cur[0], cur[1], cur[2]);
#pragma unroll
          for (int col = NEED_X2 ? 0 : 1; col < 3; ++col) {
            o[col] = short_tap2(h2[col], h1[col], cur[col], w[col][0], w[col][1], w[col][2]);
            h2[col] = h1[col];
            h1[col] = cur[col];
          }
          S.ug[row][pp] = __hmul2(o[1], o[2]);
          if constexpr (NEED_X2) S.x2g[row][pp] = o[0];
        }
      }
    }
    __syncthreads();
    for (int i = tid; i < WORDS; i += HCL_CG) {  // z history for the next tile
      const uint32_t a0 = n >= 2 ? zt[n - 2][i] : S.zh[1][i];
      const uint32_t a1 = zt[n - 1][i];
      S.zh[0][i] = a0;
      S.zh[1][i] = a1;
    }
    const bf16* ug = reinterpret_cast<const bf16*>(&S.ug[0][0]);
    const bf16* xg = reinterpret_cast<const bf16*>(&S.x2g[0][0]);
    for (int row = 0; row < n; ++row)
      fn(t0 + row, NEED_X2 ? ldbf(xg + row * HCL_CG + tid) : 0.0f, ldbf(ug + row * HCL_CG + tid));
    __syncthreads();
  }
  cp_async_wait<0>();
}

__device__ __forceinline__ void load_pole_pairs(const hyena_layer_params& P, int h, f2* p2) {
  const float* lp = P.log_poles + (long long)h * P.lp_stride_h;
#pragma unroll
  for (int i = 0; i < HCL_S / 2; ++i)
    p2[i] = f2_make(expf(lp[(2 * i) * P.lp_stride_s]), expf(lp[(2 * i + 1) * P.lp_stride_s]));
}

// modal_readout16 on mode pairs (s2[i] = modes 2i, 2i+1): the same halving tree.
__device__ __forceinline__ float readout_pairs(const f2* s2, const f2* r2) {
  f2 p[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = f2_mul(s2[i], r2[i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = f2_add(p[i], p[i + 4]);
#pragma unroll
  for (int i = 0; i < 2; ++i) p[i] = f2_add(p[i], p[i + 2]);
  const float2 v = f2_split(f2_add(p[0], p[1]));
  return add_rn(v.x, v.y);
}

__global__ void __launch_bounds__(HCL_CG)
hcl_aggregate_kernel(const hyena_layer_params P, const hyena_prefill_args A, HclWorkspace W) {
  pdl_entry();
  extern __shared__ __align__(16) uint8_t hcl_smem[];
  HclTile& S = *reinterpret_cast<HclTile*>(hcl_smem);
  ChunkCtx c;
  if (!chunk_ctx(A, W.chunk_base, blockIdx.x, c)) return;
  if (c.k == c.nch - 1) return;  // the final chunk's aggregate is never needed
  const int c0 = blockIdx.y * HCL_CG;
  const int h = c0 + threadIdx.x;
  if (c.init && (c.blk < 0 || c.blk >= A.conv_state.num_blocks)) c.init = false;
  f2 p2[HCL_S / 2], acc[HCL_S / 2];
  load_pole_pairs(P, h, p2);
#pragma unroll
  for (int i = 0; i < HCL_S / 2; ++i) acc[i] = 0ull;
  walk_chunk<false>(A, P, c, c0, S, [&](int, float, float u) {
    const f2 uu = f2_make(u, u);
#pragma unroll
    for (int i = 0; i < HCL_S / 2; ++i) acc[i] = f2_add(f2_mul(acc[i], p2[i]), uu);
  });
  f2* dst = reinterpret_cast<f2*>(W.states + ((long long)blockIdx.x * P.H + h) * HCL_S);
#pragma unroll
  for (int i = 0; i < HCL_S / 2; ++i) dst[i] = acc[i];
}

// One thread per (segment, channel, mode): S_in for every chunk, written over
// the chunk's aggregate.
__global__ void __launch_bounds__(128)
hcl_carry_kernel(const hyena_layer_params P, const hyena_prefill_args A, HclWorkspace W) {
  pdl_entry();
  const int j = blockIdx.x;
  const long long idx = (long long)blockIdx.y * 128 + threadIdx.x;  // h * 16 + s
  if (idx >= (long long)P.H * HCL_S) return;
  const int h = (int)(idx / HCL_S), s = (int)(idx % HCL_S);
  const int base = __ldg(W.chunk_base + j);
  const int nch = __ldg(W.chunk_base + j + 1) - base;
  if (nch <= 0) return;
  const long long blk = __ldg(A.state_indices + (long long)j * A.state_indices_stride);
  bool init = A.has_initial_state != nullptr && __ldg(A.has_initial_state + j) != 0;
  if (init && (blk < 0 || blk >= A.inner_state.num_blocks)) {
    flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    init = false;
  }
  const float* s2 = static_cast<const float*>(A.inner_state.data);
  float S = init ? s2[blk * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
                      (long long)s * A.inner_state.col_stride]
                 : 0.0f;
  const float pc = expf(P.log_poles[(long long)h * P.lp_stride_h + s * P.lp_stride_s] * (float)HCL_C);
  float* slot = W.states + (long long)base * P.H * HCL_S + idx;
  const long long stride = (long long)P.H * HCL_S;
  // Eight chunks per round: their aggregates are loaded together (every slot
  // is read before this thread overwrites it), then the carry runs through
  // them in order.  The last chunk's aggregate is never read.
  constexpr int CB = 8;
  for (int k0 = 0; k0 < nch; k0 += CB) {
    float a[CB];
#pragma unroll
    for (int u = 0; u < CB; ++u) a[u] = (k0 + u < nch - 1) ? slot[(k0 + u) * stride] : 0.0f;
#pragma unroll
    for (int u = 0; u < CB; ++u) {
      const int k = k0 + u;
      if (k >= nch) break;
      slot[k * stride] = S;
      if (k < nch - 1) S = add_rn(mul_rn(pc, S), a[u]);
    }
  }
}

__global__ void __launch_bounds__(HCL_CG)
hcl_output_kernel(const hyena_layer_params P, const hyena_prefill_args A, HclWorkspace W) {
  pdl_entry();
  extern __shared__ __align__(16) uint8_t hcl_smem[];
  HclTile& S = *reinterpret_cast<HclTile*>(hcl_smem);
  ChunkCtx c;
  if (!chunk_ctx(A, W.chunk_base, blockIdx.x, c)) return;
  const int c0 = blockIdx.y * HCL_CG;
  const int h = c0 + threadIdx.x;
  const bool blk_ok = c.blk >= 0 && c.blk < A.inner_state.num_blocks &&
                      c.blk < A.conv_state.num_blocks;
  if (c.init && !blk_ok) c.init = false;
  f2 p2[HCL_S / 2], r2[HCL_S / 2], s2[HCL_S / 2];
  load_pole_pairs(P, h, p2);
  {
    const float* rr = P.residues + (long long)h * P.res_stride_h;
#pragma unroll
    for (int i = 0; i < HCL_S / 2; ++i)
      r2[i] = f2_make(rr[(2 * i) * P.res_stride_s], rr[(2 * i + 1) * P.res_stride_s]);
    const f2* src = reinterpret_cast<const f2*>(W.states + ((long long)blockIdx.x * P.H + h) * HCL_S);
#pragma unroll
    for (int i = 0; i < HCL_S / 2; ++i) s2[i] = src[i];
  }
  const bf16* Dg = static_cast<const bf16*>(P.D);
  const float d = Dg ? ldbf(Dg + h) : 0.0f;
  bf16* out = static_cast<bf16*>(A.out);
  walk_chunk<true>(A, P, c, c0, S, [&](int row, float x2, float u) {
    const f2 uu = f2_make(u, u);
#pragma unroll
    for (int i = 0; i < HCL_S / 2; ++i) s2[i] = f2_add(f2_mul(s2[i], p2[i]), uu);
    float y = bf16r(readout_pairs(s2, r2));
    if (Dg) y = bf16r(y + bf16r(u * d));
    out[(long long)row * A.ldo + h] = __float2bfloat16_rn(bf16r(y * x2));
  });
  if (c.k == c.nch - 1) {
    if (!blk_ok) {
      if (threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
      return;
    }
    float* st = static_cast<float*>(A.inner_state.data);
#pragma unroll
    for (int i = 0; i < HCL_S / 2; ++i) {
      const long long b = c.blk * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride;
      const float2 v = f2_split(s2[i]);
      st[b + (long long)(2 * i) * A.inner_state.col_stride] = v.x;
      st[b + (long long)(2 * i + 1) * A.inner_state.col_stride] = v.y;
    }
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
  launch_kernel(hcl_plan_kernel, dim3(1), dim3(32), 0, st, 0u, A.query_start_loc, A.num_segments, W.chunk_base);
  int rc = check_launch("hcl_plan_kernel");
  if (rc) return rc;
  const int smem = (int)sizeof(HclTile);
  if (!smem_attr<hcl_aggregate_kernel>(smem) || !smem_attr<hcl_output_kernel>(smem))
    return fail(HYENA_ERR_CUDA, "cudaFuncSetAttribute(hcl) failed");
  launch_kernel(hcl_aggregate_kernel, dim3(max_chunks, groups), dim3(HCL_CG), (size_t)smem, st, 0u,
                P, A, W);
  if ((rc = check_launch("hcl_aggregate_kernel"))) return rc;
  launch_kernel(hcl_carry_kernel, dim3(A.num_segments, (P.H * HCL_S + 127) / 128), dim3(128), 0, st, 0u, P, A, W);
  if ((rc = check_launch("hcl_carry_kernel"))) return rc;
  launch_kernel(hcl_output_kernel, dim3(max_chunks, groups), dim3(HCL_CG), (size_t)smem, st, 0u,
                P, A, W);
  if ((rc = check_launch("hcl_output_kernel"))) return rc;
  return conv_state_update_launch(P, A, st);
}

}  // namespace hb
