// Fused Hyena FIR prefill (HCS K=7, HCM K=128) for sm_100a.
//
// One launch computes, for every packed prefill row t and channel h,
//   (x2, x1, v) = K=3 causal FIR over the in_proj triple      (vLLM causal_conv1d_fn)
//   u           = bf16(x1 * v)                                 (mixers.py:1293)
//   y           = bf16( sum_k w[h,k] * u[t-K+1+k] )            (triton_prefill.py:391-430)
//   g           = bf16(x2 * [bf16(y + bf16(D*u))  | y])        (mixers.py:1300-1302)
// with left context from the cached windows (S0 for the K=3 filter, S1 for the
// inner filter) when a segment continues a sequence, zeros otherwise.  A second
// launch writes each segment's final windows (triton_prefill.py:433-459), so no
// CTA can read a window another CTA already overwrote.
//
// Layout: a CTA owns 64 channels (192 z columns) and a contiguous range of packed
// rows, and slides along time: u values live in a shared-memory ring indexed by
// row, so the inner FIR's (K-1)-row halo is recomputed only once per CTA range
// and at segment starts, not per tile.  Every z row is read once from HBM with
// 16-byte vector loads; g is written once.
#include "common.cuh"

namespace hb {

constexpr int FIR_CG = 32;       // channels per CTA (two CTAs share an SM)
constexpr int FIR_PAIRS = FIR_CG / 2;
constexpr int FIR_BT = 128;      // rows per tile
constexpr int FIR_THREADS = 256;
constexpr int FIR_RPT = 8;       // rows per thread in the gate and tap phases
constexpr int FIR_RING = 256;    // u ring rows (power of two >= K-1 + FIR_BT)
constexpr int FIR_WORDS = 3 * FIR_PAIRS;  // bf16x2 words of z per row per CTA
constexpr int MAX_CONV_COLS = 8; // S0 window columns supported (K_short-1 + num_spec)

// z tiles in flight per CTA (one being consumed, the rest loading).  Three
// stages for K = 7 measured no faster than two (the kernel is not bound by
// bytes in flight), so both kernels use two.
template <int K>
__host__ __device__ constexpr int fir_stages() {
  return 2;
}

// Thread (pair p = tid % 16, row group g = tid / 16) owns channels c0+2p, c0+2p+1
// and tile rows 8g .. 8g+7 in both the gate and the tap phases (so the x2 it
// gates with stays in its registers).
template <int K>
struct FirShared {
  f2 ring[FIR_RING][FIR_PAIRS];                   // u by row (mod FIR_RING), fp32 pairs
  uint32_t zt[fir_stages<K>()][FIR_BT][FIR_WORDS];  // z tiles (multi-buffered), bf16x2 words
  f2 wsm[K][FIR_PAIRS];                           // inner taps as fp32 pairs, [k][pair]
  uint32_t zh[2][FIR_WORDS];             // z rows (r-2, r-1) before the tile
  bf162 sw[3][3][FIR_PAIRS];             // short taps [column x2/x1/v][tap][pair]
  bf162 dsm[FIR_PAIRS];
};

struct SegCtx {
  int a, e;       // segment rows
  long long blk;  // state block (valid only if init)
  bool init;
};

__device__ __forceinline__ SegCtx load_segment(const hyena_prefill_args& A, int j) {
  SegCtx s;
  s.a = __ldg(A.query_start_loc + j);
  s.e = __ldg(A.query_start_loc + j + 1);
  s.blk = __ldg(A.state_indices + (long long)j * A.state_indices_stride);
  s.init = A.has_initial_state != nullptr && __ldg(A.has_initial_state + j) != 0;
  return s;
}

// z value of row t, column col (absolute z column), honouring the segment's
// left context: rows before the segment come from the cached S0 window.
__device__ __forceinline__ float z_at(const hyena_prefill_args& A, const SegCtx& s, long long t,
                                      int col) {
  const bf16* z = static_cast<const bf16*>(A.z);
  if (t >= s.a) return ldbf(z + t * A.ldz + col);
  if (!s.init) return 0.0f;
  const long long back = s.a - t;  // 1 = newest cached input, in column 1
  if (back > 2) return 0.0f;
  const bf16* s0 = static_cast<const bf16*>(A.conv_state.data);
  return ldbf(s0 + s.blk * A.conv_state.block_stride + (2 - back) * A.conv_state.col_stride +
              (long long)col * A.conv_state.dim_stride);
}

// u = bf16(x1 * v) of row t >= s.a for channel h, straight from global memory
// (used for halos only).
__device__ __forceinline__ float u_at(const hyena_prefill_args& A, const hyena_layer_params& P,
                                      const SegCtx& s, long long t, int h) {
  const bf16* sw = static_cast<const bf16*>(P.short_w);
  float val[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int col = 3 * h + 1 + q;
    val[q] = short_tap(z_at(A, s, t - 2, col), z_at(A, s, t - 1, col), z_at(A, s, t, col),
                       ldbf(sw + col * 3), ldbf(sw + col * 3 + 1), ldbf(sw + col * 3 + 2));
  }
  return bf16r(val[0] * val[1]);
}

__device__ __forceinline__ uint32_t bf16_bits(float v) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// The interleaved triple words of one channel pair -> (x2, x1, v) bf16x2 pairs.
// Words: w0 = (x2_a, x1_a), w1 = (v_a, x2_b), w2 = (x1_b, v_b).
__device__ __forceinline__ void split_triples(uint32_t w0, uint32_t w1, uint32_t w2, bf162& x2,
                                              bf162& x1, bf162& v) {
  x2 = as_bf162(__byte_perm(w0, w1, 0x7610));
  x1 = as_bf162(__byte_perm(w0, w2, 0x5432));
  v = as_bf162(__byte_perm(w1, w2, 0x7610));
}

// Tiles walk the CTA's rows [r0, r1) and never straddle a segment boundary.
struct TileIt {
  int r, n, j;
};

__device__ __forceinline__ TileIt tile_at(const hyena_prefill_args& A, int r, int r1, int j) {
  const int nseg = A.num_segments;
  while (j < nseg && __ldg(A.query_start_loc + j + 1) <= r) ++j;
  TileIt t;
  t.r = r;
  t.j = j;
  t.n = (j < nseg && r < r1) ? min(FIR_BT, min(__ldg(A.query_start_loc + j + 1), r1) - r) : 0;
  return t;
}

// Issues tile t's z rows into buffer buf and closes one cp.async group (empty
// when t.n == 0, so that every loop iteration commits exactly one group).
template <int K>
__device__ __forceinline__ void prefetch_tile(FirShared<K>& S, const hyena_prefill_args& A,
                                              const TileIt& t, int buf, int c0) {
  const bf16* z = static_cast<const bf16*>(A.z);
  constexpr int VPR = FIR_WORDS * 4 / 16;  // 16-byte vectors per row
  for (int i = threadIdx.x; i < t.n * VPR; i += FIR_THREADS) {
    const int row = i / VPR, v = i % VPR;
    cp_async16(reinterpret_cast<uint4*>(&S.zt[buf][row][0]) + v,
               reinterpret_cast<const uint4*>(z + (long long)(t.r + row) * A.ldz + 3 * c0) + v);
  }
  cp_async_commit();
}

template <int K>
__global__ void __launch_bounds__(FIR_THREADS, 2)
fir_prefill_kernel(const hyena_layer_params P, const hyena_prefill_args A, int rows_per_cta) {
  pdl_entry();
  constexpr int HIST = K - 1;
  static_assert(HIST + FIR_BT <= FIR_RING, "ring too small");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FirShared<K>& S = *reinterpret_cast<FirShared<K>*>(smem_raw);

  const int tid = threadIdx.x;
  const int c0 = blockIdx.y * FIR_CG;
  const int nseg = A.num_segments;
  const int32_t* qsl = A.query_start_loc;
  const int T_end = min(A.T, __ldg(qsl + nseg));
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(T_end, r0 + rows_per_cta);
  if (r0 >= r1) return;

  bf16* out = static_cast<bf16*>(A.out);
  const bf16* iw = static_cast<const bf16*>(P.inner_w);
  const bf16* swg = static_cast<const bf16*>(P.short_w);
  const bf16* Dg = static_cast<const bf16*>(P.D);
  const float* s1 = static_cast<const float*>(A.inner_state.data);

  constexpr int NST = fir_stages<K>();
  TileIt t = tile_at(A, r0, r1, find_segment(qsl, nseg, r0));
  int buf = 0;
  TileIt pf = t;  // the last tile put in flight
  prefetch_tile(S, A, pf, 0, c0);
#pragma unroll
  for (int s = 1; s < NST - 1; ++s) {
    pf = tile_at(A, pf.r + pf.n, r1, pf.j);
    prefetch_tile(S, A, pf, s, c0);
  }

  for (int i = tid; i < K * FIR_PAIRS; i += FIR_THREADS) {
    const int k = i / FIR_PAIRS, pp = i % FIR_PAIRS;
    const long long h = c0 + 2 * pp;
    S.wsm[k][pp] = f2_make(
        __bfloat162float(iw[h * P.inner_w_stride_h + (long long)k * P.inner_w_stride_k]),
        __bfloat162float(iw[(h + 1) * P.inner_w_stride_h + (long long)k * P.inner_w_stride_k]));
  }
  for (int i = tid; i < 9 * FIR_PAIRS; i += FIR_THREADS) {
    const int col = i / (3 * FIR_PAIRS), tap = (i / FIR_PAIRS) % 3, pp = i % FIR_PAIRS;
    const long long h = c0 + 2 * pp;
    S.sw[col][tap][pp] = __halves2bfloat162(swg[(3 * h + col) * 3 + tap],
                                            swg[(3 * (h + 1) + col) * 3 + tap]);
  }
  if (tid < FIR_PAIRS)
    S.dsm[tid] = Dg ? __halves2bfloat162(Dg[c0 + 2 * tid], Dg[c0 + 2 * tid + 1])
                    : __floats2bfloat162_rn(0.f, 0.f);

  const int pp = tid % FIR_PAIRS;  // channel pair
  const int rg = tid / FIR_PAIRS;  // row group 0..15 (FIR_BT / FIR_RPT)
  float* ring_f = reinterpret_cast<float*>(&S.ring[0][0]);
  int cur_seg = -1;

  while (t.n > 0) {
    const TileIt nt = tile_at(A, t.r + t.n, r1, t.j);
    // the tile NST-1 ahead goes into the buffer the previous tile has released
    pf = tile_at(A, pf.r + pf.n, r1, pf.j);
    prefetch_tile(S, A, pf, (buf + NST - 1) % NST, c0);

    if (t.j != cur_seg) {
      // ---- new segment (or the CTA's first rows): history rows [r-HIST, r) and z rows r-2, r-1
      cur_seg = t.j;
      SegCtx seg = load_segment(A, t.j);
      if (seg.init && (seg.blk < 0 || seg.blk >= A.inner_state.num_blocks ||
                       seg.blk >= A.conv_state.num_blocks)) {
        if (tid == 0) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
        seg.init = false;
      }
      __syncthreads();  // previous tile's readers of ring / zh are done
      for (int i = tid; i < HIST * FIR_CG; i += FIR_THREADS) {
        const int m = i / FIR_CG + 1, cc = i % FIR_CG;
        const long long tr = (long long)t.r - m;
        float val;
        if (tr >= seg.a) {
          val = u_at(A, P, seg, tr, c0 + cc);
        } else if (seg.init && seg.a - tr <= HIST) {
          const long long col = HIST - (seg.a - tr);
          val = s1[seg.blk * A.inner_state.block_stride + col * A.inner_state.col_stride +
                   (long long)(c0 + cc) * A.inner_state.dim_stride];
        } else {
          val = 0.0f;
        }
        ring_f[(int)(tr & (FIR_RING - 1)) * FIR_CG + cc] = val;
      }
      for (int i = tid; i < 2 * FIR_WORDS; i += FIR_THREADS) {
        const int q = i / FIR_WORDS, wd = i % FIR_WORDS;
        const long long tr = (long long)t.r - 2 + q;
        const uint32_t lo = bf16_bits(z_at(A, seg, tr, 3 * c0 + 2 * wd));
        const uint32_t hi = bf16_bits(z_at(A, seg, tr, 3 * c0 + 2 * wd + 1));
        S.zh[q][wd] = lo | (hi << 16);
      }
    }
    cp_async_wait<NST - 1>();  // this tile's group (one group is committed per tile)
    __syncthreads();

    const int n = t.n, r = t.r;
    // ---- K=3 short filter on channel pairs, sliding over 8 consecutive rows
    const int g0 = rg * FIR_RPT;
    bf162 x2r[FIR_RPT];
    if (g0 < n) {
      bf162 w[3][3];
#pragma unroll
      for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int k = 0; k < 3; ++k) w[c][k] = S.sw[c][k][pp];
      bf162 h2[3], h1[3];
      {
        const uint32_t* a = g0 >= 2 ? &S.zt[buf][g0 - 2][3 * pp] : &S.zh[g0][3 * pp];
        const uint32_t* b = g0 >= 1 ? &S.zt[buf][g0 - 1][3 * pp] : &S.zh[1][3 * pp];
        split_triples(a[0], a[1], a[2], h2[0], h2[1], h2[2]);
        split_triples(b[0], b[1], b[2], h1[0], h1[1], h1[2]);
      }
#pragma unroll
      for (int i = 0; i < FIR_RPT; ++i) {
        const int row = g0 + i;
        if (row < n) {
          bf162 cur[3], o[3];
          split_triples(S.zt[buf][row][3 * pp], S.zt[buf][row][3 * pp + 1],
                        S.zt[buf][row][3 * pp + 2], cur[0], cur[1], cur[2]);
#pragma unroll
          for (int c = 0; c < 3; ++c) {
            o[c] = short_tap2(h2[c], h1[c], cur[c], w[c][0], w[c][1], w[c][2]);
            h2[c] = h1[c];
            h1[c] = cur[c];
          }
          S.ring[(r + row) & (FIR_RING - 1)][pp] = f2_from_bf162(__hmul2(o[1], o[2]));
          x2r[i] = o[0];
        }
      }
    }
    __syncthreads();

    // ---- z history for the next tile (reads zt/zh only; ring untouched)
    if (tid < FIR_WORDS) {
      uint32_t h0v, h1v;
      if (n >= 2) {
        h0v = S.zt[buf][n - 2][tid];
        h1v = S.zt[buf][n - 1][tid];
      } else {
        h0v = S.zh[1][tid];
        h1v = S.zt[buf][0][tid];
      }
      S.zh[0][tid] = h0v;
      S.zh[1][tid] = h1v;
    }

    // ---- inner FIR over the ring: thread = (channel pair, rows i0..i0+7)
    const int i0 = rg * FIR_RPT;
    if (i0 < n) {
      f2 acc[FIR_RPT];
#pragma unroll
      for (int q = 0; q < FIR_RPT; ++q) acc[q] = 0ull;  // +0.0f in both lanes
      const int base = r + i0 - HIST;  // may be negative: masked arithmetic wraps
      f2 cur[8], nxt[8];
#pragma unroll
      for (int x = 0; x < 8; ++x) cur[x] = S.ring[(base + x) & (FIR_RING - 1)][pp];
#pragma unroll
      for (int kb = 0; kb < K; kb += 8) {
#pragma unroll
        for (int x = 0; x < 8; ++x)
          if (kb + 8 + x < HIST + FIR_RPT) nxt[x] = S.ring[(base + kb + 8 + x) & (FIR_RING - 1)][pp];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          if (kb + kk < K) {
            const f2 wv = S.wsm[kb + kk][pp];
#pragma unroll
            for (int q = 0; q < FIR_RPT; ++q)
              acc[q] = f2_fma(wv, (q + kk < 8) ? cur[q + kk] : nxt[q + kk - 8], acc[q]);
          }
        }
#pragma unroll
        for (int x = 0; x < 8; ++x) cur[x] = nxt[x];
      }
      const bool has_d = Dg != nullptr;
      const bf162 d2 = S.dsm[pp];
      bf162* outp = reinterpret_cast<bf162*>(out + (long long)(r + i0) * A.ldo + c0) + pp;
      const long long ld2 = A.ldo / 2;
#pragma unroll
      for (int q = 0; q < FIR_RPT; ++q) {
        if (i0 + q < n) {
          bf162 y = bf162_from_f2(acc[q]);
          if (has_d)
            y = __hadd2(y, __hmul2(d2, bf162_from_f2(S.ring[(r + i0 + q) & (FIR_RING - 1)][pp])));
          outp[q * ld2] = __hmul2(x2r[q], y);
        }
      }
    }
    __syncthreads();
    buf = (buf + 1) % NST;
    t = nt;
  }
}

// Second launch: each segment's final windows.  S0 columns 0..1 <- last two z
// values of concat(old S0[:, 0:2] | zeros, z_seg) (mixers.py:374, 380-382; any
// speculative columns 2..W0-1 are left as they are); S1[:, :K-1] <- last K-1 u
// values of concat(old S1 | zeros, u_seg) (triton_prefill.py:433-459).
// K == 0 updates S0 only.
template <int K>
__global__ void __launch_bounds__(128)
prefill_state_kernel(const hyena_layer_params P, const hyena_prefill_args A) {
  pdl_entry();
  const int j = blockIdx.x;
  const int h = blockIdx.y * 128 + threadIdx.x;
  if (h >= P.H) return;
  SegCtx seg = load_segment(A, j);
  const int L = seg.e - seg.a;
  if (L <= 0) return;
  if (seg.blk < 0 || seg.blk >= A.conv_state.num_blocks ||
      (K > 0 && seg.blk >= A.inner_state.num_blocks)) {
    if (threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    return;
  }
  bf16* s0 = static_cast<bf16*>(A.conv_state.data);
  const bf16* z = static_cast<const bf16*>(A.z);
  // blockIdx.z splits the K-1 history positions when every one of them comes
  // from this segment's own z rows (L >= K+1: no old window is read, so the
  // split blocks are independent); otherwise block z = 0 does all of them, in
  // the in-place order below.  Only block z = 0 reads and rewrites S0.
  const int zi = (int)blockIdx.z;

  // Old S0 columns 0..1 for the three z columns of channel h (read before any write).
  float old0[3][2];
#pragma unroll
  for (int q = 0; q < 3; ++q)
#pragma unroll
    for (int i = 0; i < 2; ++i)
      old0[q][i] = seg.init && zi == 0 ? ldbf(s0 + seg.blk * A.conv_state.block_stride +
                                   (long long)i * A.conv_state.col_stride +
                                   (long long)(3 * h + q) * A.conv_state.dim_stride)
                            : 0.0f;

  if constexpr (K > 0) {
    constexpr int HIST = K - 1;
    float* s1 = static_cast<float*>(A.inner_state.data);
    const bf16* sw = static_cast<const bf16*>(P.short_w);
    float w1[3], w2[3];
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      w1[q] = ldbf(sw + (3 * h + 1) * 3 + q);
      w2[q] = ldbf(sw + (3 * h + 2) * 3 + q);
    }
    float* base = s1 + seg.blk * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride;
    const bool split = L >= HIST + 2;
    const int chunk = (HIST + (int)gridDim.z - 1) / (int)gridDim.z;
    const int i0 = split ? zi * chunk : (zi == 0 ? 0 : HIST);
    const int i1 = split ? min(HIST, i0 + chunk) : HIST;
    for (int i = i0; i < i1; ++i) {
      const int src = L + i;  // position in concat(hist[HIST], u[L])
      float val;
      if (src < HIST) {
        val = seg.init ? base[(long long)src * A.inner_state.col_stride] : 0.0f;
      } else {
        const long long t = (long long)seg.a + (src - HIST);
        float xv[2][3];
#pragma unroll
        for (int m = 0; m < 3; ++m) {
          const long long tt = t - 2 + m;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            float v;
            if (tt >= seg.a) {
              v = ldbf(z + tt * A.ldz + 3 * h + 1 + q);
            } else {
              const int back = int(seg.a - tt);  // 1..2
              v = back == 1 ? old0[1 + q][1] : old0[1 + q][0];
            }
            xv[q][m] = v;
          }
        }
        const float x1 = short_tap(xv[0][0], xv[0][1], xv[0][2], w1[0], w1[1], w1[2]);
        const float vv = short_tap(xv[1][0], xv[1][1], xv[1][2], w2[0], w2[1], w2[2]);
        val = bf16r(x1 * vv);
      }
      base[(long long)i * A.inner_state.col_stride] = val;
    }
  }

  // New S0 columns 0..1.
  if (zi != 0) return;
#pragma unroll
  for (int q = 0; q < 3; ++q) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int src = L + i;  // position in concat(old[0:2], z[L])
      const float val = src < 2 ? old0[q][src]
                                : ldbf(z + (long long)(seg.a + src - 2) * A.ldz + 3 * h + q);
      s0[seg.blk * A.conv_state.block_stride + (long long)i * A.conv_state.col_stride +
         (long long)(3 * h + q) * A.conv_state.dim_stride] = __float2bfloat16_rn(val);
    }
  }
}

// ---------------------------------------------------------------- launchers
template <int K>
static int launch_fir(const hyena_layer_params& P, const hyena_prefill_args& A, cudaStream_t st) {
  const size_t smem = sizeof(FirShared<K>);
  if (!smem_attr<fir_prefill_kernel<K>>((int)smem))
    return fail(HYENA_ERR_CUDA, "cudaFuncSetAttribute(fir_prefill) failed");
  // Rows per CTA: long enough that the (K-1)-row halo is a small fraction,
  // short enough to fill the 148 SMs several times over.
  const int groups = P.H / FIR_CG;
  int rows = K > 16 ? 2048 : 1024;
  const long long want_ctas = 148LL * 8;
  while (rows > FIR_BT && (long long)((A.T + rows - 1) / rows) * groups < want_ctas) rows /= 2;
  dim3 grid((A.T + rows - 1) / rows, groups);
  launch_kernel(fir_prefill_kernel<K>, dim3(grid), dim3(FIR_THREADS), smem, st, 0u, P, A, rows);
  int rc = check_launch("fir_prefill_kernel");
  if (rc) return rc;
  dim3 g2(A.num_segments, (P.H + 127) / 128, K > 16 ? 8 : 1);
  launch_kernel(prefill_state_kernel<K>, dim3(g2), dim3(128), 0, st, 0u, P, A);
  return check_launch("prefill_state_kernel");
}

int fir_prefill_launch(const hyena_layer_params& P, const hyena_prefill_args& A, cudaStream_t st) {
  if (P.K == 128) return launch_fir<128>(P, A, st);
  if (P.K == 7) return launch_fir<7>(P, A, st);
  return fail(HYENA_ERR_UNSUPPORTED, "FIR prefill supports K = 7 or 128");
}

int conv_state_update_launch(const hyena_layer_params& P, const hyena_prefill_args& A,
                             cudaStream_t st) {
  dim3 g2(A.num_segments, (P.H + 127) / 128);
  launch_kernel(prefill_state_kernel<0>, dim3(g2), dim3(128), 0, st, 0u, P, A);
  return check_launch("prefill_state_kernel<0>");
}

}  // namespace hb
