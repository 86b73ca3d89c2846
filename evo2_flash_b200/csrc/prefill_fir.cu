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
// Layout: a CTA owns 16 channels (48 z columns) and a contiguous range of packed
// rows, and slides along time in tiles of 256 rows:
//   gate phase   z tile (cp.async, 3 stages) -> K=3 filter, x1*v on CUDA cores;
//                u goes to a per-channel, time-major bf16 buffer in shared memory,
//                x2 stays in registers;
//   tap phase    the inner FIR as a banded Toeplitz product on the tensor cores
//                (mma.sync m16n8k16, bf16 x bf16 -> fp32): per channel,
//                Y(i, j) = y[t0 + 32 j + i] = sum_d W(i, d) U(d, j) with
//                W(i, d) = w[d - i + K - 1] (the taps, zero outside [0, K)) and
//                U(d, j) = u[t0 + 32 j + d].  W is fixed per channel and lives in
//                registers as A fragments; the second 16-row M tile (i + 16) is
//                the first one shifted by one k-step, so it reuses the same
//                fragments.  U fragments come from that buffer with ldmatrix;
//                results go back through stmatrix.trans into a per-channel,
//                time-major y tile;
//   store phase  + D*u, * x2, bf16 rounding as torch does, coalesced rows of g.
// bf16 x bf16 products are exact in fp32, so the tensor-core form differs from
// the reference's oldest-first fp32 sum only in the order of the additions.
// The inner FIR's (K-1)-row halo is recomputed once per CTA range and at segment
// starts.  Every z row is read once from HBM; g is written once.
//
// Shared-memory layouts avoid bank conflicts for every access pattern used:
// per channel, u (halo + tile) and the y tile are stored as lines of 32 rows
// with an 80-byte pitch (five 16-byte chunks, one of them padding) and an odd
// per-channel chunk stride, so the eight row addresses of an ldmatrix /
// stmatrix phase (rows 32 apart: chunks 5 apart) and the chunk pairs of the
// gate and store phases fall on eight different bank groups, and every
// ldmatrix address is a per-lane base plus a compile-time offset.  After each
// tile its last HALO rows of u move to the front as the next tile's history.
// z rows carry an 8-word gap after every 8 rows so that the four row groups of
// a warp read disjoint banks.
#include "common.cuh"

namespace hb {

constexpr int FIR_CG = 16;       // channels per CTA
constexpr int FIR_PAIRS = FIR_CG / 2;
constexpr int FIR_BT = 256;      // rows per tile
constexpr int FIR_THREADS = 256;
constexpr int FIR_WARPS = FIR_THREADS / 32;
constexpr int FIR_RPT = 8;       // rows per thread in the gate and store phases
constexpr int FIR_WORDS = 3 * FIR_PAIRS;                       // bf16x2 z words per row
constexpr int FIR_ZT_WORDS = FIR_WORDS * FIR_BT + 8 * (FIR_BT / 8);  // one z tile
constexpr int FIR_YS_CH = (FIR_BT / 32) * 5 + 1;  // y tile chunks per channel (odd stride)
constexpr int FIR_WOFF = 64;     // zero padding in front of the staged taps
constexpr int FIR_STAGES = 3;    // z tiles in flight per CTA

static_assert(FIR_PAIRS * (FIR_BT / FIR_RPT) == FIR_THREADS, "gate mapping");
static_assert(2 * FIR_WARPS == FIR_CG, "two channels per warp in the tap phase");

// u rows kept per channel: HALO rows of history (the tap phase reads from
// d = -HALO) and the tile.
template <int K>
struct FirGeom {
  static constexpr int HALO = 16 * ((K - 1 + 15) / 16);
  static constexpr int LINES = (HALO + FIR_BT + 31) / 32;
  static constexpr int UCH = (LINES * 5) | 1;  // 16-byte chunks per channel (odd stride)
};

template <int K>
struct FirShared {
  uint32_t zt[FIR_STAGES][FIR_ZT_WORDS];  // z tiles, bf16x2 words
  uint4 ub[FIR_CG * FirGeom<K>::UCH];     // u by (channel, row), bf16
  // y tile by (channel, tile row); before the first tile it holds the taps,
  // zero-padded, from which each warp builds its A fragments.
  union {
    uint4 ys[FIR_CG * FIR_YS_CH];
    bf16 wpad[FIR_CG][K + 128];
  };
  uint32_t zh[2][2][FIR_WORDS];          // z rows (r-2, r-1) before the tile, [tile parity]
  bf162 sw[3][3][FIR_PAIRS];             // short taps [column x2/x1/v][tap][pair]
  bf162 dsm[FIR_PAIRS];
};

// Word offset of z tile row r (an 8-word gap after every 8 rows).
__device__ __forceinline__ int zrow(int r) { return r * FIR_WORDS + 8 * (r >> 3); }

// 16-byte chunk holding row t (t % 8 == 0: rows t..t+7) of one channel in a
// line-padded per-channel array (32 rows per 80-byte line).
__device__ __forceinline__ int line_chunk(int t) { return 5 * (t >> 5) + ((t & 31) >> 3); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(p))
               : "memory");
}
__device__ __forceinline__ void stsm_x4_trans(void* p, uint32_t r0, uint32_t r1, uint32_t r2,
                                              uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(
                   smem_u32(p)),
               "r"(r0), "r"(r1), "r"(r2), "r"(r3)
               : "memory");
}
// d += a . b, m16n8k16, bf16 operands, fp32 accumulators.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(bf16 lo, bf16 hi) {
  return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}
__device__ __forceinline__ uint32_t pack_rn(float lo, float hi) {
  return as_u32(__floats2bfloat162_rn(lo, hi));
}

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
// (used for halos only); w1 / w2: the x1 and v columns' short taps.
__device__ __forceinline__ float u_at(const hyena_prefill_args& A, const SegCtx& s, long long t,
                                      int h, const float (&w1)[3], const float (&w2)[3]) {
  const int col = 3 * h + 1;
  const float x1 = short_tap(z_at(A, s, t - 2, col), z_at(A, s, t - 1, col), z_at(A, s, t, col),
                             w1[0], w1[1], w1[2]);
  const float vv = short_tap(z_at(A, s, t - 2, col + 1), z_at(A, s, t - 1, col + 1),
                             z_at(A, s, t, col + 1), w2[0], w2[1], w2[2]);
  return bf16r(x1 * vv);
}

__device__ __forceinline__ uint32_t bf16_bits(float v) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// The interleaved triple words of one channel pair -> (x2, x1, v) bf16x2 pairs.
// Words: w0 = (x2_a, x1_a), w1 = (v_a, x2_b), w2 = (x1_b, v_b).
__device__ __forceinline__ bf162 split_x2(uint32_t w0, uint32_t w1) {
  return as_bf162(__byte_perm(w0, w1, 0x7610));
}
__device__ __forceinline__ void split_x1v(uint32_t w0, uint32_t w1, uint32_t w2, bf162& x1,
                                          bf162& v) {
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
// Thread (group gi, row rin, chunk v) copies rows 8 gi + rin + 40 k: row
// offsets in the gapped tile then advance by a constant.
template <int K>
__device__ __forceinline__ void prefetch_tile(FirShared<K>& S, const hyena_prefill_args& A,
                                              const TileIt& t, int buf, int c0) {
  constexpr int VPR = FIR_WORDS * 4 / 16;                      // 16-byte chunks per row
  constexpr int PASS = (FIR_THREADS / (8 * VPR)) * 8;          // rows per pass
  constexpr int DST_STEP = PASS * FIR_WORDS + 8 * (PASS / 8);  // zrow(r + PASS) - zrow(r)
  const int tid = threadIdx.x;
  if (tid < PASS * VPR) {
    const int v = tid % VPR;
    int r = 8 * (tid / (8 * VPR)) + (tid % (8 * VPR)) / VPR;
    uint32_t* dst = &S.zt[buf][zrow(r) + 4 * v];
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const bf16*>(A.z) +
                                                      (long long)(t.r + r) * A.ldz + 3 * c0) + v;
    const long long step = (long long)PASS * A.ldz / 8;  // in 16-byte units
    for (; r < t.n; r += PASS, dst += DST_STEP, src += step) cp_async16(dst, src);
  }
  cp_async_commit();
}

template <int K>
__global__ void __launch_bounds__(FIR_THREADS, 2)
fir_prefill_kernel(const hyena_layer_params P, const hyena_prefill_args A, int rows_per_cta) {
  pdl_entry();
  constexpr int HIST = K - 1;
  constexpr int KB = (HIST + 15) / 16;  // k-steps of U below d = 0
  constexpr int NKS = KB + 2;           // k-steps of U: d in [DB0, 32)
  constexpr int NA = NKS - 1;           // distinct W fragments
  constexpr int DB0 = -16 * KB;
  using G = FirGeom<K>;
  static_assert(G::HALO == -DB0, "history rows");
  static_assert(sizeof(bf16) * FIR_CG * (K + 128) <= sizeof(uint4) * FIR_CG * FIR_YS_CH,
                "tap staging must fit in the y tile");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FirShared<K>& S = *reinterpret_cast<FirShared<K>*>(smem_raw);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * FIR_CG;
  const int nseg = A.num_segments;
  const int32_t* qsl = A.query_start_loc;
  const int T_end = min(A.T, __ldg(qsl + nseg));
  const int r0 = blockIdx.y * rows_per_cta;
  const int r1 = min(T_end, r0 + rows_per_cta);
  if (r0 >= r1) return;

  bf16* out = static_cast<bf16*>(A.out);
  const bf16* iw = static_cast<const bf16*>(P.inner_w);
  const bf16* swg = static_cast<const bf16*>(P.short_w);
  const bf16* Dg = static_cast<const bf16*>(P.D);
  const float* s1 = static_cast<const float*>(A.inner_state.data);

  TileIt t = tile_at(A, r0, r1, find_segment(qsl, nseg, r0));
  int buf = 0;
  TileIt pf = t;  // the last tile put in flight
  prefetch_tile(S, A, pf, 0, c0);
#pragma unroll
  for (int s = 1; s < FIR_STAGES - 1; ++s) {
    pf = tile_at(A, pf.r + pf.n, r1, pf.j);
    prefetch_tile(S, A, pf, s, c0);
  }

  // ---- parameters: taps (zero-padded), short taps, D; the u buffer starts at zero
  for (int i = tid; i < FIR_CG * (K + 128); i += FIR_THREADS) {
    const int ch = i % FIR_CG, e = i / FIR_CG - FIR_WOFF;  // channel-fastest: coalesced taps
    S.wpad[ch][e + FIR_WOFF] =
        (e >= 0 && e < K)
            ? iw[(long long)(c0 + ch) * P.inner_w_stride_h + (long long)e * P.inner_w_stride_k]
            : __float2bfloat16_rn(0.0f);
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
  for (int i = tid; i < FIR_CG * G::UCH; i += FIR_THREADS) S.ub[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();

  // ---- W fragments of this warp's two channels (A operand of m16n8k16):
  // a0a1 (i = g, d0 + {0,1}), a2a3 (i = g + 8, d0 + {0,1}), a4a5 / a6a7 the same at d0 + 8,
  // with d0 = DB0 + 16 ks + 2q.  W(i, d) depends on d - i only, so with
  // word(m) = (W(g, DB0 + 2q + 8 (m - 1)), the next tap): a0a1 = a6a7 = word(2 ks + 1),
  // a2a3 = word(2 ks), a4a5 = word(2 ks + 2); NW distinct words cover every k-step.
  constexpr int NW = 2 * NA + 1;
  uint32_t wv[2][NW];
  {
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const bf16* wc = &S.wpad[2 * warp + cc][FIR_WOFF + K - 1];  // wc[d - i] = W(i, d)
#pragma unroll
      for (int m = 0; m < NW; ++m) {
        const int off = DB0 + 2 * q - g + 8 * (m - 1);
        wv[cc][m] = pack_bf16(wc[off], wc[off + 1]);
      }
    }
  }

  // gate / store mapping: an 8-lane phase holds 4 channel pairs x 2 row groups
  const int pp = (lane & 3) | ((lane >> 1) & 4);
  const int rg = warp * 4 + (((lane >> 2) & 1) | ((lane >> 3) & 2));
  const int g0 = rg * FIR_RPT;
  bf16* ub_h = reinterpret_cast<bf16*>(S.ub);
  int cur_seg = -1;
  int zc = 0;  // the zh buffer holding the current tile's z history

  while (t.n > 0) {
    const TileIt nt = tile_at(A, t.r + t.n, r1, t.j);
    __syncthreads();  // the previous tile is finished: u buffer, y tile, z buffer, zh
    // the tile FIR_STAGES-1 ahead goes into the buffer the previous tile released
    pf = tile_at(A, pf.r + pf.n, r1, pf.j);
    prefetch_tile(S, A, pf, (buf + FIR_STAGES - 1) % FIR_STAGES, c0);

    if (t.j != cur_seg) {
      // ---- new segment (or the CTA's first rows): history rows [r-HIST, r) and z rows r-2, r-1
      cur_seg = t.j;
      SegCtx seg = load_segment(A, t.j);
      if (seg.init && (seg.blk < 0 || seg.blk >= A.inner_state.num_blocks ||
                       seg.blk >= A.conv_state.num_blocks)) {
        if (tid == 0) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
        seg.init = false;
      }
      for (int i = tid; i < HIST * FIR_CG; i += FIR_THREADS) {
        const int m = i / FIR_CG + 1, cc = i % FIR_CG;
        const long long tr = (long long)t.r - m;
        float val;
        if (tr >= seg.a) {
          float w1[3], w2[3];  // the pair's short taps, from shared memory
#pragma unroll
          for (int k = 0; k < 3; ++k) {
            const float2 a1 = __bfloat1622float2(S.sw[1][k][cc >> 1]);
            const float2 a2 = __bfloat1622float2(S.sw[2][k][cc >> 1]);
            w1[k] = (cc & 1) ? a1.y : a1.x;
            w2[k] = (cc & 1) ? a2.y : a2.x;
          }
          val = u_at(A, seg, tr, c0 + cc, w1, w2);
        } else if (seg.init && seg.a - tr <= HIST) {
          const long long col = HIST - (seg.a - tr);
          val = s1[seg.blk * A.inner_state.block_stride + col * A.inner_state.col_stride +
                   (long long)(c0 + cc) * A.inner_state.dim_stride];
        } else {
          val = 0.0f;
        }
        const int tr_rel = G::HALO - m;  // buffer row of input row t.r - m
        ub_h[(cc * G::UCH + line_chunk(tr_rel & ~7)) * 8 + (tr_rel & 7)] = __float2bfloat16_rn(val);
      }
      for (int i = tid; i < 2 * FIR_WORDS; i += FIR_THREADS) {
        const int q = i / FIR_WORDS, wd = i % FIR_WORDS;
        const long long tr = (long long)t.r - 2 + q;
        const uint32_t lo = bf16_bits(z_at(A, seg, tr, 3 * c0 + 2 * wd));
        const uint32_t hi = bf16_bits(z_at(A, seg, tr, 3 * c0 + 2 * wd + 1));
        S.zh[zc][q][wd] = lo | (hi << 16);
      }
    }
    cp_async_wait<FIR_STAGES - 1>();  // this tile's group (one group is committed per tile)
    __syncthreads();

    const int n = t.n, r = t.r;
    const uint32_t* zt = S.zt[buf];
    // rows g0 - 2, g0 - 1 of this thread's channel pair (z history at g0 = 0)
    const uint32_t* zga = g0 >= 2 ? &zt[zrow(g0 - 2) + 3 * pp] : &S.zh[zc][g0][3 * pp];
    const uint32_t* zgb = g0 >= 1 ? &zt[zrow(g0 - 1) + 3 * pp] : &S.zh[zc][1][3 * pp];
    const uint32_t* zg = &zt[zrow(g0) + 3 * pp];  // rows g0.. of one 8-row group
    // ---- gate phase: K=3 short filter of the x1 and v columns on a channel pair
    // over 8 consecutive rows, u = x1 * v (x2 is filtered in the store phase)
    if (g0 < n) {
      bf162 w[2][3];
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int k = 0; k < 3; ++k) w[c][k] = S.sw[c + 1][k][pp];
      bf162 h2[2], h1[2];
      split_x1v(zga[0], zga[1], zga[2], h2[0], h2[1]);
      split_x1v(zgb[0], zgb[1], zgb[2], h1[0], h1[1]);
      uint32_t uu[FIR_RPT];
#pragma unroll
      for (int i = 0; i < FIR_RPT; ++i) {
        const uint32_t* zr = zg + i * FIR_WORDS;
        bf162 cur[2], o[2];
        split_x1v(zr[0], zr[1], zr[2], cur[0], cur[1]);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          o[c] = short_tap2(h2[c], h1[c], cur[c], w[c][0], w[c][1], w[c][2]);
          h2[c] = h1[c];
          h1[c] = cur[c];
        }
        // rows past the tile read stale shared memory: their u must not reach the buffer
        uu[i] = g0 + i < n ? as_u32(__hmul2(o[0], o[1])) : 0u;
      }
      // channel pairs by row -> 8 consecutive rows per channel
      uint4 ua, ub;
      ua.x = __byte_perm(uu[0], uu[1], 0x5410); ub.x = __byte_perm(uu[0], uu[1], 0x7632);
      ua.y = __byte_perm(uu[2], uu[3], 0x5410); ub.y = __byte_perm(uu[2], uu[3], 0x7632);
      ua.z = __byte_perm(uu[4], uu[5], 0x5410); ub.z = __byte_perm(uu[4], uu[5], 0x7632);
      ua.w = __byte_perm(uu[6], uu[7], 0x5410); ub.w = __byte_perm(uu[6], uu[7], 0x7632);
      S.ub[2 * pp * G::UCH + line_chunk(G::HALO + g0)] = ua;
      S.ub[(2 * pp + 1) * G::UCH + line_chunk(G::HALO + g0)] = ub;
    }
    __syncthreads();

    // ---- tap phase: per channel, Y (32 x 8) = W (32 x 16 NKS) . U (16 NKS x 8)
    {
      // ldmatrix rows: U(d, j) for j = lane & 7 at d = DB0 + 16 ks + 8 ((lane >> 3) & 1),
      // buffer row HALO + 32 j + d = 32 j + 16 ks + 8 ((lane >> 3) & 1)
      const int lbase = 5 * (lane & 7) + ((lane >> 3) & 1);
      // stmatrix.trans rows: matrix k = (M tile m, half h), row q = column j of Y:
      // tile rows 32 q + 16 m + 8 h
      const int sk = lane >> 3, sq = lane & 7;
      const int sbase = 5 * sq + 2 * (sk >> 1) + (sk & 1);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int ch = 2 * warp + cc;
        float acc[2][4];
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[m][e] = 0.0f;
        // every U fragment of the channel in flight before the first product
        uint32_t bu[NKS][2];
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks)
          ldsm_x2(bu[ks][0], bu[ks][1], &S.ub[ch * G::UCH + lbase + 5 * (ks >> 1) + 2 * (ks & 1)]);
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks) {
          const uint32_t b0 = bu[ks][0], b1 = bu[ks][1];
          if (ks < NA) {
            const uint32_t a[4] = {wv[cc][2 * ks + 1], wv[cc][2 * ks], wv[cc][2 * ks + 2],
                                   wv[cc][2 * ks + 1]};
            mma_bf16(acc[0], a, b0, b1);
          }
          if (ks >= 1) {
            const uint32_t a[4] = {wv[cc][2 * ks - 1], wv[cc][2 * ks - 2], wv[cc][2 * ks],
                                   wv[cc][2 * ks - 1]};
            mma_bf16(acc[1], a, b0, b1);
          }
        }
        stsm_x4_trans(&S.ys[ch * FIR_YS_CH + sbase], pack_rn(acc[0][0], acc[0][1]),
                      pack_rn(acc[0][2], acc[0][3]), pack_rn(acc[1][0], acc[1][1]),
                      pack_rn(acc[1][2], acc[1][3]));
      }
    }
    __syncthreads();

    // ---- store phase: g = bf16(x2 * bf16(y + bf16(D * u))) on channel pairs
    if (g0 < n) {
      const uint4 ya = S.ys[2 * pp * FIR_YS_CH + line_chunk(g0)];
      const uint4 yb = S.ys[(2 * pp + 1) * FIR_YS_CH + line_chunk(g0)];
      const uint32_t yaw[4] = {ya.x, ya.y, ya.z, ya.w}, ybw[4] = {yb.x, yb.y, yb.z, yb.w};
      uint32_t uaw[4] = {0, 0, 0, 0}, ubw[4] = {0, 0, 0, 0};
      const bool has_d = Dg != nullptr;
      if (has_d) {
        const uint4 ua = S.ub[2 * pp * G::UCH + line_chunk(G::HALO + g0)];
        const uint4 ub = S.ub[(2 * pp + 1) * G::UCH + line_chunk(G::HALO + g0)];
        uaw[0] = ua.x; uaw[1] = ua.y; uaw[2] = ua.z; uaw[3] = ua.w;
        ubw[0] = ub.x; ubw[1] = ub.y; ubw[2] = ub.z; ubw[3] = ub.w;
      }
      const bf162 d2 = S.dsm[pp];
      const bf162 wx0 = S.sw[0][0][pp], wx1 = S.sw[0][1][pp], wx2 = S.sw[0][2][pp];
      bf162 x2h2 = split_x2(zga[0], zga[1]), x2h1 = split_x2(zgb[0], zgb[1]);
      bf162* outp = reinterpret_cast<bf162*>(out + (long long)(r + g0) * A.ldo + c0) + pp;
      const long long ld2 = A.ldo / 2;
#pragma unroll
      for (int i = 0; i < FIR_RPT; ++i) {
        const bf162 x2c = split_x2(zg[i * FIR_WORDS], zg[i * FIR_WORDS + 1]);
        const bf162 x2 = short_tap2(x2h2, x2h1, x2c, wx0, wx1, wx2);
        x2h2 = x2h1;
        x2h1 = x2c;
        if (g0 + i < n) {
          const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
          bf162 y = as_bf162(__byte_perm(yaw[i >> 1], ybw[i >> 1], sel));
          // D*u is rounded to bf16 before the add, as torch does: the _rn
          // multiply keeps the compiler from fusing the two into one bf16 FMA
          if (has_d) y = __hadd2(y, __hmul2_rn(d2, as_bf162(__byte_perm(uaw[i >> 1], ubw[i >> 1], sel))));
          outp[i * ld2] = __hmul2(x2, y);
        }
      }
    }
    // ---- z history for the next tile of this segment, into the other zh
    // buffer (the store phase may still read this tile's)
    if (tid < FIR_WORDS) {
      uint32_t h0v, h1v;
      if (n >= 2) {
        h0v = zt[zrow(n - 2) + tid];
        h1v = zt[zrow(n - 1) + tid];
      } else {
        h0v = S.zh[zc][1][tid];
        h1v = zt[zrow(0) + tid];
      }
      S.zh[zc ^ 1][0][tid] = h0v;
      S.zh[zc ^ 1][1][tid] = h1v;
    }
    zc ^= 1;
    // ---- the tile's last HALO rows of u become the next tile's history
    // (read from rows the store phase does not touch; written over rows no
    // one reads until the next tile's tap phase)
    for (int i = tid; i < FIR_CG * (G::HALO / 8); i += FIR_THREADS) {
      const int cc = i / (G::HALO / 8), c8 = 8 * (i % (G::HALO / 8));
      S.ub[cc * G::UCH + line_chunk(c8)] = S.ub[cc * G::UCH + line_chunk(FIR_BT + c8)];
    }
    buf = (buf + 1) % FIR_STAGES;
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
  // Rows per CTA: a multiple of the tile, long enough that the (K-1)-row halo is
  // a small fraction, short enough to fill the 148 SMs several times over.  A
  // CTA whose rows start inside a segment recomputes the halo's u from z with
  // scalar loads: at the config-2 shape (8 x 8192 rows, H = 4096) 8192-row
  // CTAs, which start at segment starts, took HCM 0.884 -> 0.800 ms and HCS
  // 0.610 -> 0.588 ms against 4096 rows (2048 rows: 1.037 / 0.656 ms).
  const int groups = P.H / FIR_CG;
  int rows = 8192;
  const long long want_ctas = 148LL * 8;
  while (rows > FIR_BT && (long long)((A.T + rows - 1) / rows) * groups < want_ctas) rows /= 2;
  while ((A.T + rows - 1) / rows > 65535) rows *= 2;
  // channel groups fastest: CTAs that run together read neighbouring 96-byte
  // pieces of the same z rows
  dim3 grid(groups, (A.T + rows - 1) / rows);
  launch_kernel(fir_prefill_kernel<K>, dim3(grid), dim3(FIR_THREADS), smem, st, 0u, P, A, rows);
  int rc = check_launch("fir_prefill_kernel");
  if (rc) return rc;
  dim3 g2(A.num_segments, (P.H + 127) / 128, K > 16 ? 8 : 1);
  launch_kernel(prefill_state_kernel<K>, dim3(g2), dim3(128), 0, st, 0u, P, A);
  return check_launch("prefill_state_kernel");
}

int fir_prefill_launch(const hyena_layer_params& P, const hyena_prefill_args& A, cudaStream_t st) {
  if (P.H % FIR_CG != 0) return fail(HYENA_ERR_INVALID, "FIR prefill needs H % 16 == 0");
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
