// tcgen05 GEMM family for sm_100a.
//
// Persistent CTAs (two per SM) walk 128 x BN output tiles with a warp-specialised pipeline:
// gather warps build the A operand by implicit im2col from fp32 activations (converted to
// fp16 with round-to-nearest-even, as the reference's dk_im2col_half does) or a TMA warp
// loads fp16 rows; the TMA warp loads B tiles; one thread issues tcgen05.mma into a TMEM
// accumulator that is double-buffered, so the epilogue warps (TMEM -> registers -> fused
// bias / GELU / GLU / residual / layout transform -> global) of one tile overlap the loads
// and MMAs of the next.  Operands use the K-major SWIZZLE_128B layout (see umma.cuh); a
// ring of shared-memory stages with mbarrier full/empty pairs feeds the MMAs.
//
// The same kernels serve dk_gemm_half (backend.h:117-122), the implicit-GEMM convolutions
// (replacing im2col + GEMM + bias, ops.c:31-77), the stride-phase transposed convolutions
// (replacing transpose + GEMM + col2im, ops.c:143-177) and the transformer linears
// (ops.c:234-257 and the head split of attn.cu:60-89).  A CUDA-core kernel with identical
// semantics handles calls the TMA path cannot express (unaligned pointers or strides) and
// backs the "simt" option used for A/B checks.
#include <cudaTypedefs.h>

#include "gemm.cuh"
#include "umma.cuh"

namespace dcb {

constexpr int kBM = 128, kBK = 64;
constexpr uint32_t kATileBytes = kBM * kBK * 2;

struct Shape {
  int M, N, K;  // rows of the UMMA A operand, rows of the B operand, reduction length
  int nkb;      // K blocks of 64
  int stages;
  int a_shared, b_shared;
  int mtiles, ntiles, batch;  // output tiles of 128 x BN per batch entry
};

// ------------------------------------------------------------- epilogue
struct RowInfo {
  int64_t base;  // output offset of the row (conv modes)
  int ho, wo;
  int b, t;      // heads mode
};

static __device__ __forceinline__ RowInfo decode_row(const Epi &e, int64_t m) {
  RowInfo ri{0, 0, 0, 0, 0};
  if (e.mode == EPI_CONV || e.mode == EPI_CONVTR) {
    int64_t hw = (int64_t)e.Ho * e.Wo;
    int64_t n = m / hw, rem = m - n * hw;
    ri.ho = (int)(rem / e.Wo);
    ri.wo = (int)(rem - (int64_t)ri.ho * e.Wo);
    int64_t n1 = n / e.oN2, n2 = n - n1 * e.oN2;
    ri.base = n1 * e.oN1 + n2 * e.oN2s;
  } else if (e.mode == EPI_HEADS) {
    ri.b = (int)(m / e.T);
    ri.t = (int)(m - (int64_t)ri.b * e.T);
  }
  return ri;
}

// store one accumulator element (every mode except GLU), m/n in UMMA coordinates
static __device__ __forceinline__ void store_elem(const Epi &e, const Shape &s, int bz,
                                                  int64_t m, int64_t n, const RowInfo &ri,
                                                  float v) {
  switch (e.mode) {
    case EPI_GEMM: {
      int64_t idx = e.swapped ? (int64_t)bz * e.strideC + n * e.ldc + m
                              : (int64_t)bz * e.strideC + m * e.ldc + n;
      float r = e.alpha * v;
      if (e.beta != 0.f) r += e.beta * e.C[idx];
      e.C[idx] = r;
      break;
    }
    case EPI_CONV: {
      if (n >= e.O) return;
      float val = v + (e.bias ? e.bias[n] : 0.f);
      if (e.act == 1) val = gelu_f(val);
      int64_t off = ri.base + n * e.oC + (int64_t)ri.ho * e.oH + ri.wo;
      if (e.res) val = e.res[off] + e.scale[n] * val;
      e.y[off] = val;
      break;
    }
    case EPI_CONVTR: {
      // columns are (phase r, channel o), channels fastest
      int r = (int)(n / e.O), o = (int)(n - (int64_t)r * e.O);
      if (r >= e.stride) return;
      int q = e.axis_h ? ri.ho : ri.wo;
      int t = q * e.stride + r - e.crop;
      if (t < 0 || t >= e.out_len) return;
      float val = v + (e.bias ? e.bias[o] : 0.f);
      if (e.act == 1) val = gelu_f(val);
      int64_t off = ri.base + (int64_t)o * e.oC +
                    (e.axis_h ? (int64_t)t * e.oH + ri.wo : (int64_t)ri.ho * e.oH + t);
      e.y[off] = val;
      break;
    }
    case EPI_ROWS_F32: {
      float val = v + (e.bias ? e.bias[n] : 0.f);
      if (e.act == 1) val = gelu_f(val);
      if (e.res) val = e.res[m * e.ldr + n] + e.gamma[n] * val;
      ((float *)e.out)[m * e.ldo + n] = val;
      break;
    }
    case EPI_ROWS_F16: {
      float val = v + (e.bias ? e.bias[n] : 0.f);
      if (e.act == 1) val = gelu_f(val);
      ((uint16_t *)e.out)[m * e.ldo + n] = f2h_bits(val);
      break;
    }
    case EPI_HEADS: {
      int sec = (int)(n / e.sec_cols);
      int cc = (int)(n - (int64_t)sec * e.sec_cols);
      int h = cc / e.hd, d = cc - h * e.hd;
      float val = v + (e.bias ? e.bias[n] : 0.f);
      uint16_t hv = f2h_bits(val);
      int64_t bh = (int64_t)ri.b * e.heads + h;
      if (e.sec_layout[sec] == 0) {
        e.sec_ptr[sec][(bh * e.T + ri.t) * e.hd + d] = hv;
      } else {
        e.sec_ptr[sec][(bh * e.hd + d) * e.Tp + ri.t] = hv;
      }
      break;
    }
    default:
      break;
  }
}

// GLU pair (a = column c of the tile's first half, b = same column of the second half)
static __device__ __forceinline__ void store_glu(const Epi &e, int64_t o, const RowInfo &ri,
                                                 float va, float vb, int64_t img) {
  if (o >= e.O) return;
  float a = va + (e.bias ? e.bias[o] : 0.f);
  float b = vb + (e.bias ? e.bias[e.O + o] : 0.f);
  if (e.act == 3) {
    const float mu = e.gn_mean[img], rs = e.gn_rstd[img];
    a = (a - mu) * rs * e.gn_w[o] + e.gn_b[o];
    b = (b - mu) * rs * e.gn_w[e.O + o] + e.gn_b[e.O + o];
  }
  float val = a * sigmoid_f(b);
  int64_t off = ri.base + o * e.oC + (int64_t)ri.ho * e.oH + ri.wo;
  if (e.res) val = e.res[off] + e.scale[o] * val;
  e.y[off] = val;
}

// 16 consecutive accumulator columns of one row: vectorised stores where the layout allows
// (e.vec, checked on the host), element stores otherwise
static __device__ __forceinline__ void store_chunk16(const Epi &e, const Shape &s, int bz,
                                                     int64_t m, int64_t n0, const RowInfo &ri,
                                                     const float (&v)[16]) {
  if (e.vec && n0 + 16 <= s.N) {
    if (e.mode == EPI_ROWS_F32) {
      float o[16];
#pragma unroll
      for (int i = 0; i < 16; i++) {
        float val = v[i] + (e.bias ? e.bias[n0 + i] : 0.f);
        if (e.act == 1) val = gelu_f(val);
        o[i] = val;
      }
      if (e.res) {
        const float4 *rp = (const float4 *)(e.res + m * e.ldr + n0);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float4 r = rp[j];
          o[4 * j] = r.x + e.gamma[n0 + 4 * j] * o[4 * j];
          o[4 * j + 1] = r.y + e.gamma[n0 + 4 * j + 1] * o[4 * j + 1];
          o[4 * j + 2] = r.z + e.gamma[n0 + 4 * j + 2] * o[4 * j + 2];
          o[4 * j + 3] = r.w + e.gamma[n0 + 4 * j + 3] * o[4 * j + 3];
        }
      }
      float4 *op = (float4 *)((float *)e.out + m * e.ldo + n0);
#pragma unroll
      for (int j = 0; j < 4; j++)
        op[j] = make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
      return;
    }
    if (e.mode == EPI_ROWS_F16 || e.mode == EPI_HEADS) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        float a = v[i] + (e.bias ? e.bias[n0 + i] : 0.f);
        float b = v[i + 1] + (e.bias ? e.bias[n0 + i + 1] : 0.f);
        if (e.act == 1) {
          a = gelu_f(a);
          b = gelu_f(b);
        }
        w[i >> 1] = pack_h2(a, b);
      }
      uint16_t *dst;
      if (e.mode == EPI_ROWS_F16) {
        dst = (uint16_t *)e.out + m * e.ldo + n0;
      } else {
        // a 16-column chunk lies inside one section and one head (hd % 16 == 0)
        const int sec = (int)(n0 / e.sec_cols);
        const int cc = (int)(n0 - (int64_t)sec * e.sec_cols);
        const int h = cc / e.hd, d0 = cc - h * e.hd;
        const int64_t bh = (int64_t)ri.b * e.heads + h;
        if (e.sec_layout[sec] != 0) {
          uint16_t *col = e.sec_ptr[sec] + (bh * e.hd + d0) * e.Tp + ri.t;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            col[(2 * i) * e.Tp] = (uint16_t)(w[i] & 0xffffu);
            col[(2 * i + 1) * e.Tp] = (uint16_t)(w[i] >> 16);
          }
          return;
        }
        dst = e.sec_ptr[sec] + (bh * e.T + ri.t) * e.hd + d0;
      }
      uint4 *dp = (uint4 *)dst;
      dp[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dp[1] = make_uint4(w[4], w[5], w[6], w[7]);
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 16; i++) {
    if (n0 + i < s.N) store_elem(e, s, bz, m, n0 + i, ri, v[i]);
  }
}

// ------------------------------------------------------------- tensor-core kernel
// Persistent: each CTA walks output tiles blockIdx.x, +gridDim.x, ... (N tiles fastest, so
// a gathered A row block is re-read from L1/L2 while it is hot).  Warp roles:
//   warps 0-3 (0-7 without a gather)  epilogue: TMEM lane quarter (warp & 3); with 8 warps
//                                     warp >> 2 picks the half of the tile's columns;
//   warps 4-7 (gather only)            A producers: one tile row per thread, 64 K columns
//                                     per stage (implicit im2col, fp32 -> fp16 RNE);
//   warp 8                             TMA: B tiles (and A tiles when A is fp16 rows);
//   warp 9                             TMEM allocation; lane 0 issues tcgen05.mma.
// The accumulator is double-buffered in TMEM for N tiles up to 128 columns, so the
// epilogue of tile i overlaps the operand loads and MMAs of tile i+1.
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;

template <int BN, bool GATHER>
struct UmmaCfg {
  static constexpr int kEpiWarps = GATHER ? 4 : 8;
  static constexpr int kBufs = BN <= 128 ? 2 : 1;
  static constexpr int kAccCols = BN < 32 ? 32 : BN;
  static constexpr int kTmemCols = kAccCols * kBufs;  // a power of two >= 32
  static constexpr uint32_t kBTileBytes = BN * 128;
  static constexpr int kStageFloats = GATHER ? 4 * 32 * 32 : 0;  // per-warp transposes
};

static __device__ __forceinline__ void tile_coords(const Shape &s, int64_t tile, int &bz,
                                                   int64_t &m0, int &nt) {
  const int64_t per_b = (int64_t)s.mtiles * s.ntiles;
  bz = (int)(tile / per_b);
  const int64_t rem = tile - (int64_t)bz * per_b;
  const int64_t mt = rem / s.ntiles;
  nt = (int)(rem - mt * s.ntiles);
  m0 = mt * kBM;
}

// Epilogue of one 128 x BN accumulator tile (TMEM columns from `tacc`) by NW warps: warp w
// reads TMEM lane quarter (w & 3); with NW == 8, w >> 2 picks the half of the columns.
// Rows r >= row_lim of the tile are outside the output.  EPI_CONV goes through `wst`, this
// warp's [CW columns][32 rows] transpose buffer, so that lane l stores rows 4(l & 7)..+3 of
// one channel with a 16-byte store; other modes store per row (store_chunk16).
// 16 consecutive column constants p[0..15] (16-byte aligned): four 16-byte loads of one
// address per lane, served by the L1 broadcast
static __device__ __forceinline__ void ld_cols16(const float *p, float (&d)[16]) {
  const float4 *p4 = (const float4 *)p;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float4 t = __ldg(p4 + j);
    d[4 * j] = t.x;
    d[4 * j + 1] = t.y;
    d[4 * j + 2] = t.z;
    d[4 * j + 3] = t.w;
  }
}

// Row-mode epilogue (EPI_ROWS_F32 / EPI_ROWS_F16 / EPI_HEADS) for 16-byte aligned outputs
// and column constants (e.cvec, checked on the host): bias / gamma and the residual row
// are loaded while the accumulator load is in flight.
// e.row_stats in row mode: add a warp's output sums to their groups of e.stat_rows rows
// (fp32 per lane over its columns, fp64 across lanes) in this CTA's slot; one atomic pair
// per warp when all its valid rows share a group, per lane otherwise
static __device__ __forceinline__ void rows_stats_add(const Epi &e, bool mv, int64_t m,
                                                      float ls, float lq) {
  const int lane = threadIdx.x & 31;
  double *st = e.row_stats + 2 * (blockIdx.x % kStatSlots);
  const unsigned valid = __ballot_sync(0xffffffffu, mv);
  if (!valid) return;
  const int64_t g = mv ? m / e.stat_rows : -1;
  const int64_t g0 = __shfl_sync(0xffffffffu, g, __ffs(valid) - 1);
  if (__all_sync(0xffffffffu, !mv || g == g0)) {
    double s = mv ? (double)ls : 0.0, q = mv ? (double)lq : 0.0;
    for (int o = 16; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      q += __shfl_xor_sync(0xffffffffu, q, o);
    }
    if (lane == 0) {
      atomicAdd(&st[2 * kStatSlots * g0], s);
      atomicAdd(&st[2 * kStatSlots * g0 + 1], q);
    }
  } else if (mv) {
    atomicAdd(&st[2 * kStatSlots * g], (double)ls);
    atomicAdd(&st[2 * kStatSlots * g + 1], (double)lq);
  }
}

template <int BN, int NW>
static __device__ __forceinline__ void rows_epi_fast(const Shape &s, const Epi &e,
                                                     uint32_t trow, int half, int r, int64_t m,
                                                     int n0, int row_lim) {
  const bool mv = r < row_lim;
  const RowInfo ri = mv ? decode_row(e, m) : RowInfo{0, 0, 0, 0, 0};
  constexpr int PER = NW == 8 ? (BN / 2 < 16 ? 16 : BN / 2) : BN;
  const int cbeg = NW == 8 ? half * PER : 0;
  float ls = 0.f, lq = 0.f;  // e.row_stats: this lane's sums over its columns
  for (int c0 = cbeg; c0 < cbeg + PER && c0 < BN; c0 += 16) {
    const int64_t n = (int64_t)n0 + c0;
    if (n >= s.N) break;
    float v[16], bb[16];
    tmem_ld16(trow + c0, v);
    if (e.bias) {
      ld_cols16(e.bias + n, bb);
    } else {
#pragma unroll
      for (int i = 0; i < 16; i++) bb[i] = 0.f;
    }
    if (e.mode == EPI_ROWS_F32) {
      float rr[16], gg[16];
      if (e.res) {
        ld_cols16(e.gamma + n, gg);
        if (mv) {
          const float4 *rp = (const float4 *)(e.res + m * e.ldr + n);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const float4 t = rp[j];
            rr[4 * j] = t.x;
            rr[4 * j + 1] = t.y;
            rr[4 * j + 2] = t.z;
            rr[4 * j + 3] = t.w;
          }
        }
      }
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) v[i] += bb[i];
      if (e.act == 1) {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = gelu_f(v[i]);
      }
      if (e.res) {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = fmaf(gg[i], v[i], rr[i]);
      }
      if (mv) {
        float4 *op = (float4 *)((float *)e.out + m * e.ldo + n);
#pragma unroll
        for (int j = 0; j < 4; j++)
          op[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        if (e.row_stats) {
          const int nv = s.N - n < 16 ? (int)(s.N - n) : 16;
#pragma unroll
          for (int i = 0; i < 16; i++) {
            if (i < nv) {
              ls += v[i];
              lq = fmaf(v[i], v[i], lq);
            }
          }
        }
      }
    } else {
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) v[i] += bb[i];
      if (e.act == 1) {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = gelu_f(v[i]);
      }
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; i++) w[i] = pack_h2(v[2 * i], v[2 * i + 1]);
      if (mv) {
        uint16_t *dst;
        if (e.mode == EPI_ROWS_F16) {
          dst = (uint16_t *)e.out + m * e.ldo + n;
        } else {
          // EPI_HEADS: a 16-column chunk lies inside one section and one head
          const int sec = (int)(n / e.sec_cols);
          const int cc = (int)(n - (int64_t)sec * e.sec_cols);
          const int h = cc / e.hd, d0 = cc - h * e.hd;
          const int64_t bh = (int64_t)ri.b * e.heads + h;
          if (e.sec_layout[sec] != 0) {
            uint16_t *col = e.sec_ptr[sec] + (bh * e.hd + d0) * e.Tp + ri.t;
#pragma unroll
            for (int i = 0; i < 8; i++) {
              col[(2 * i) * e.Tp] = (uint16_t)(w[i] & 0xffffu);
              col[(2 * i + 1) * e.Tp] = (uint16_t)(w[i] >> 16);
            }
            continue;
          }
          dst = e.sec_ptr[sec] + (bh * e.T + ri.t) * e.hd + d0;
        }
        uint4 *dp = (uint4 *)dst;
        dp[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dp[1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
  }
  if (e.mode == EPI_ROWS_F32 && e.row_stats) rows_stats_add(e, mv, m, ls, lq);
}

template <int BN, int NW, int CW, int EK>
static __device__ __forceinline__ void epilogue_tile(const Shape &s, const Epi &e, uint32_t tacc,
                                                     int warp, int lane, int bz, int64_t m0,
                                                     int nt, int row_lim, float *wst) {
  const int quarter = warp & 3, half = NW == 8 ? (warp >> 2) : 0;
  const int r = quarter * 32 + lane;
  const uint32_t trow = tacc + ((uint32_t)(quarter * 32) << 16);
  const int n0 = nt * BN;
  const int64_t m = m0 + r;
  if constexpr (EK == 1) {
    rows_epi_fast<BN, NW>(s, e, trow, half, r, m, n0, row_lim);
  } else if (e.mode == EPI_CONV && wst) {
    const int rq = 4 * (lane & 7);
    int64_t poff[4];
    bool pv[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      pv[i] = quarter * 32 + rq + i < row_lim;
      poff[i] = 0;
      if (pv[i]) {
        const RowInfo ri = decode_row(e, m0 + quarter * 32 + rq + i);
        poff[i] = ri.base + (int64_t)ri.ho * e.oH + ri.wo;
      }
    }
    const bool contig = pv[3] && poff[1] == poff[0] + 1 && poff[2] == poff[0] + 2 &&
                        poff[3] == poff[0] + 3;
    const bool glu = e.act >= 2;
    // act 3: GroupNorm statistics of this lane's row (one image per Ho * Wo rows)
    float gmu = 0.f, grs = 0.f;
    if (e.act == 3 && r < row_lim) {
      const int64_t img = m / ((int64_t)e.Ho * e.Wo);
      gmu = e.gn_mean[img];
      grs = e.gn_rstd[img];
    }
    const int ncols = glu ? e.glu_half : BN;
    const int per = NW == 8 ? (ncols >= 32 ? ncols / 2 : (half == 0 ? ncols : 0)) : ncols;
    const int cbeg = NW == 8 && ncols >= 32 ? half * per : 0;
    const int obase = glu ? nt * e.glu_half : n0;
    for (int c0 = cbeg; c0 < cbeg + per; c0 += CW) {
      const int cw = cbeg + per - c0 >= CW ? CW : 16;
      for (int sub = 0; sub < cw; sub += 16) {
        float va[16];
        tmem_ld16(trow + c0 + sub, va);
        if (glu) {
          float vb[16];
          tmem_ld16(trow + e.glu_half + c0 + sub, vb);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int o = obase + c0 + sub + i;
            float val = 0.f;
            if (o < e.O) {
              float a = va[i] + (e.bias ? e.bias[o] : 0.f);
              float b = vb[i] + (e.bias ? e.bias[e.O + o] : 0.f);
              if (e.act == 3) {
                a = (a - gmu) * grs * e.gn_w[o] + e.gn_b[o];
                b = (b - gmu) * grs * e.gn_w[e.O + o] + e.gn_b[e.O + o];
              }
              val = a * sigmoid_f(b);
            }
            wst[(sub + i) * 32 + lane] = val;
          }
        } else {
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int o = obase + c0 + sub + i;
            float val = va[i] + ((e.bias && o < e.O) ? e.bias[o] : 0.f);
            if (e.act == 1) val = gelu_f(val);
            wst[(sub + i) * 32 + lane] = val;
          }
        }
      }
      __syncwarp();
      for (int cc = lane >> 3; cc < cw; cc += 4) {
        const int o = obase + c0 + cc;
        if (o >= e.O) continue;
        const float4 v4 = *(const float4 *)(wst + cc * 32 + rq);
        float vv[4] = {v4.x, v4.y, v4.z, v4.w};
        const int64_t a = poff[0] + (int64_t)o * e.oC;
        const uintptr_t al = (uintptr_t)(e.y + a) | (e.res ? (uintptr_t)(e.res + a) : 0);
        if (contig && (al & 15) == 0) {
          if (e.res) {
            const float4 rr = *(const float4 *)(e.res + a);
            const float sc = e.scale[o];
            vv[0] = rr.x + sc * vv[0];
            vv[1] = rr.y + sc * vv[1];
            vv[2] = rr.z + sc * vv[2];
            vv[3] = rr.w + sc * vv[3];
          }
          *(float4 *)(e.y + a) = make_float4(vv[0], vv[1], vv[2], vv[3]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; i++) {
            if (!pv[i]) continue;
            const int64_t ai = poff[i] + (int64_t)o * e.oC;
            float val = vv[i];
            if (e.res) val = e.res[ai] + e.scale[o] * val;
            e.y[ai] = val;
          }
        }
      }
      __syncwarp();
    }
  } else {
    const bool mv = r < row_lim;
    const RowInfo ri = mv ? decode_row(e, m) : RowInfo{0, 0, 0, 0, 0};
    constexpr int PER = NW == 8 ? (BN / 2 < 16 ? 16 : BN / 2) : BN;
    const int cbeg = NW == 8 ? half * PER : 0;
    for (int c0 = cbeg; c0 < cbeg + PER && c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(trow + c0, v);
      tmem_wait_ld();
      if (mv) store_chunk16(e, s, bz, m, (int64_t)n0 + c0, ri, v);
    }
  }
}

template <int BN, bool GATHER, int EK>
__global__ void __launch_bounds__(kThreads, 2)
    k_umma(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const Shape s, const Gather g, const Epi e) {
  using Cfg = UmmaCfg<BN, GATHER>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int stages = s.stages;
  uint8_t *sA = smem;
  uint8_t *sB = smem + stages * kATileBytes;
  float *stg = (float *)(sB + stages * Cfg::kBTileBytes);
  uint64_t *full = (uint64_t *)(stg + Cfg::kStageFloats);
  uint64_t *empty = full + stages;
  uint64_t *acc_full = empty + stages;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *fin = acc_empty + 2;
  uint32_t *tslot = (uint32_t *)(fin + 1);
  int2 *ktab = (int2 *)(tslot + 2);

  // a fault recorded by an earlier kernel: end this grid at once (uniform CTA decision)
  __shared__ uint32_t s_abort;
  if (threadIdx.x == 0) s_abort = fault_pending() ? 1u : 0u;
  __syncthreads();
  if (s_abort) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles_total = (int64_t)s.mtiles * s.ntiles * s.batch;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; i++) {
      mbar_init(&full[i], 1 + (GATHER ? 4 : 0));
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], Cfg::kEpiWarps);
    }
    mbar_init(fin, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tslot, (uint32_t)Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (GATHER) {
    const int nk = s.nkb * kBK;
    for (int k = threadIdx.x; k < nk; k += kThreads) {
      int2 t;
      if (k < g.K) {
        int c = k % g.C, kk = k / g.C, kh = kk / g.KW, kw = kk - kh * g.KW;
        int dh = kh * g.DH, dw = kw * g.DW;
        t.x = (int)((int64_t)c * g.sC + (int64_t)dh * g.sH + dw);
        t.y = dh | (dw << 16);
      } else {
        t.x = 0;
        t.y = 0x7fff;  // row offset out of every image: the element reads as zero
      }
      ktab[k] = t;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == kTmaWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmB);
      if (!GATHER) tma_prefetch_desc(&tmA);
      const uint32_t bytes = Cfg::kBTileBytes + (GATHER ? 0u : kATileBytes);
      uint32_t it = 0;
      int st = 0;        // ring stage of K block `it` and its phase parity (kept
      uint32_t ph = 0;   // incrementally: no division in the issue loop)
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < ntiles_total; tile += gridDim.x) {
        int bz, nt;
        int64_t m0;
        tile_coords(s, tile, bz, m0, nt);
        const int cA = s.a_shared ? 0 : bz, cB = s.b_shared ? 0 : bz;
        for (int kb = 0; kb < s.nkb; kb++, it++) {
          if (!mbar_wait(&empty[st], ph ^ 1u, kFaultEmpty)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[st], bytes);
          tma_load_3d(sB + st * Cfg::kBTileBytes, &tmB, &full[st], kb * kBK, nt * BN, cB);
          if (!GATHER)
            tma_load_3d(sA + st * kATileBytes, &tmA, &full[st], kb * kBK, (int)m0, cA);
          if (++st == stages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok && !GATHER) {
        // fault path: the last `stages` armed stages may still have copies in flight; let
        // them land before the CTA exits (each stage's latest phase completes by its own
        // transaction bytes alone when the operands come only from TMA)
        for (uint32_t j = it > (uint32_t)stages ? it - (uint32_t)stages : 0u; j < it; j++) {
          mbar_drain(&full[j % (uint32_t)stages], (j / (uint32_t)stages) & 1u);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(kBM, BN);
      uint32_t it = 0, local = 0;
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < ntiles_total; tile += gridDim.x, local++) {
        const uint32_t buf = local % (uint32_t)Cfg::kBufs;
        const uint32_t use = local / (uint32_t)Cfg::kBufs;
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, kFaultDone)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * (uint32_t)Cfg::kAccCols;
        for (int kb = 0; kb < s.nkb; kb++, it++) {
          if (!mbar_wait(&full[st], ph, kFaultFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(smem_u32(sA + st * kATileBytes));
          const uint64_t bd = sw128_desc(smem_u32(sB + st * Cfg::kBTileBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; k++) {
            // +32 bytes per K=16 step inside the 128-byte swizzle row (>> 4 = 2)
            umma_f16(d, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          if (it == 0 && *(volatile uint32_t *)&g_test_withhold != 0u &&
              atomicExch(&g_test_withhold, 0u) != 0u) {
            // test hook (option "test_withhold_arrive"): stage 0 is never released
          } else {
            umma_commit(&empty[st]);
          }
          if (++st == stages) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      // every MMA of this CTA has completed before the accumulator is released
      umma_commit(fin);
      mbar_wait(fin, 0, kFaultDone);
    }
  } else if (GATHER && warp >= 4) {
    // ---- warps 4-7: A producers, tile row r = 32 (warp - 4) + lane, all 64 K columns
    const int r = (warp - 4) * 32 + lane;
    const float *__restrict__ x = g.x;
    const float *__restrict__ x2 = g.x2;
    const int64_t hw = (int64_t)g.Ho * g.Wo;
    uint32_t it = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles_total; tile += gridDim.x) {
      int bz, nt;
      int64_t m0;
      tile_coords(s, tile, bz, m0, nt);
      const int64_t p = m0 + r;
      int64_t base = 0;
      int h0 = -(1 << 20), w0 = 0;
      if (p < s.M) {
        const int64_t n = p / hw, rem = p - n * hw;
        const int ho = (int)(rem / g.Wo), wo = (int)(rem - (int64_t)ho * g.Wo);
        const int64_t n1 = n / g.N2, n2 = n - n1 * g.N2;
        h0 = ho * g.SH - g.PH;
        w0 = wo * g.SW - g.PW;
        base = n1 * g.sN1 + n2 * g.sN2 + (int64_t)h0 * g.sH + w0;
      }
      for (int kb = 0; kb < s.nkb; kb++, it++) {
        const int st = (int)(it % (uint32_t)stages);
        const uint32_t ph = (it / (uint32_t)stages) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, kFaultEmpty)) {
          ok = false;
          break;
        }
        const int2 *kt = ktab + kb * kBK;
        const uint32_t a_base = smem_u32(sA + st * kATileBytes);
        // all 64 loads of the row are issued before the first shared-memory store
        // (predicated loads in select form, so that none waits for another)
        float v[kBK];
        if (x2) {
#pragma unroll
          for (int i = 0; i < kBK; i++) {
            const int2 t = kt[i];
            const int hh = h0 + (t.y & 0xffff), ww = w0 + (t.y >> 16);
            const bool in = (unsigned)hh < (unsigned)g.H && (unsigned)ww < (unsigned)g.W;
            v[i] = in ? __ldg(x + base + t.x) + __ldg(x2 + base + t.x) : 0.f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < kBK; i++) {
            const int2 t = kt[i];
            const int hh = h0 + (t.y & 0xffff), ww = w0 + (t.y >> 16);
            const bool in = (unsigned)hh < (unsigned)g.H && (unsigned)ww < (unsigned)g.W;
            v[i] = in ? __ldg(x + base + t.x) : 0.f;
          }
        }
#pragma unroll
        for (int c = 0; c < 8; c++) {
          st_shared_v4(a_base + sw128_off(r, c), pack_h2(v[8 * c], v[8 * c + 1]),
                       pack_h2(v[8 * c + 2], v[8 * c + 3]), pack_h2(v[8 * c + 4], v[8 * c + 5]),
                       pack_h2(v[8 * c + 6], v[8 * c + 7]));
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[st]);
      }
    }
  } else if (warp < Cfg::kEpiWarps) {
    // ---- epilogue warps: TMEM lane quarter (warp & 3) = rows 32q..32q+31 of the tile
    float *wst = stg + (warp & 3) * (32 * 32);  // [32 columns][32 rows] of this warp (conv)
    uint32_t local = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles_total; tile += gridDim.x, local++) {
      int bz, nt;
      int64_t m0;
      tile_coords(s, tile, bz, m0, nt);
      const uint32_t buf = local % (uint32_t)Cfg::kBufs;
      const uint32_t use = local / (uint32_t)Cfg::kBufs;
      if (!warp_all(mbar_wait(&acc_full[buf], use & 1u, kFaultDone))) break;
      tc_fence_after();
      const int64_t left = (int64_t)s.M - m0;
      epilogue_tile<BN, Cfg::kEpiWarps, 32, EK>(s, e, tmem + buf * (uint32_t)Cfg::kAccCols, warp,
                                            lane, bz, m0, nt, left < kBM ? (int)left : kBM,
                                            GATHER ? wst : nullptr);
      // this warp's TMEM reads are complete: release the accumulator buffer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------- TMA im2col conv kernel
// Convolutions over fp32 activations whose positions along W are contiguous (stride 1 in
// W, every other stride a multiple of 16 bytes): the freq-branch convs of the model.  A
// tile is 128 consecutive output positions of one output line (n, ho).  K runs over
// (kh, 64-channel block, kw, channel): for each (kh, channel block) the TMA warp loads
// one fp32 box x[n][c0..c0+63][h][w_al..w_al+BW) (w_al = the first input position of the
// tile rounded down to a 16-byte boundary; rows, positions and channels outside the
// tensor read as zero, which is the convolution's zero padding) that serves every W tap;
// eight converter warps turn it into one fp16 (round-to-nearest-even) K-major
// SWIZZLE_128B A tile per W tap, (one output position, 32 channels) per thread, adding the skip tensor
// when there is one; the TMA warp also streams the B tiles; one thread issues
// tcgen05.mma.  The box ring and the operand ring are separate, so a box is refilled as
// soon as its A tiles are built.  One persistent CTA per SM: 512 TMEM columns hold two
// accumulators of up to 256 columns, so the epilogue (8 warps) of a tile overlaps the
// next tile's loads and MMAs.  All rows of a tile share (n, ho): the epilogue addresses
// each output column once per tile and stores 4 consecutive positions per 16-byte store.
// Weights are in (kh, channel block, kw) order with channels zero-padded to whole blocks
// of 64: B[n][((kh * ncb + cb) * KW + kw) * 64 + c].
struct ConvTma {
  int KH, KW, SH, PH, DH, PW, DW;
  int Ho, Wo;
  int ncb;        // 64-channel blocks
  int64_t lines;  // output lines (images * Ho)
  int tpl;        // tiles of 128 positions per line
  int N2;         // images = n1 * N2 + n2
  int N, nkb, ntiles;
  int bw;         // box width (positions), a multiple of 4
  int xstages, stages;
};

constexpr int kCtThreads = 576;  // warps 0-7 epilogue, 8-15 converters, 16 TMA, 17 MMA
constexpr int kCtTmaWarp = 16, kCtMmaWarp = 17;
constexpr int kCtBoxMax = 256;   // TMA box extent limit
constexpr int kCtEpiCW = 16;     // epilogue transpose chunk (columns)

template <int BN, bool X2>
struct CtCfg {
  static constexpr uint32_t kBBytes = BN * 128;
  static constexpr uint32_t kABStage = kATileBytes + kBBytes;  // a multiple of 1024
  static constexpr int kAccCols = BN < 32 ? 32 : BN;
  static constexpr int kTmemCols = kAccCols * 2;  // two accumulators, a power of two
};

static __device__ __forceinline__ void tma_load_5d(void *dst, const CUtensorMap *map,
                                                   uint64_t *bar, int c0, int c1, int c2,
                                                   int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// sigmoid with the hardware exp2 / reciprocal approximations (relative error ~1e-6)
static __device__ __forceinline__ float sigmoid_fast(float x) {
  return __fdividef(1.0f, 1.0f + __expf(-x));
}

// tile -> (line, first position, N tile); N tiles fastest
static __device__ __forceinline__ void ct_tile(const ConvTma &c, int64_t tile, int64_t &line,
                                               int &wo0, int &nt) {
  nt = (int)(tile % c.ntiles);
  const int64_t rest = tile / c.ntiles;
  line = rest / c.tpl;
  wo0 = (int)(rest - line * c.tpl) * kBM;
}

// Epilogue of a line tile (EPI_CONV, or EPI_CONVTR along H) by 8 warps: warp w reads TMEM
// lane quarter (w & 3) = positions 32q..32q+31 and half (w >> 2) of the columns, 16
// columns per step through its [16][32] transpose buffer `wst`.
template <int BN>
static __device__ __forceinline__ void ct_epilogue(const ConvTma &c, const Epi &e, uint32_t tacc,
                                                   int warp, int lane, int64_t line, int wo0,
                                                   int nt, float *wst) {
  const int quarter = warp & 3, half = warp >> 2;
  const uint32_t trow = tacc + ((uint32_t)(quarter * 32) << 16);
  const int64_t n = line / c.Ho;
  const int ho = (int)(line - n * c.Ho);
  const int64_t n1 = n / e.oN2, n2 = n - n1 * e.oN2;
  const int64_t base = n1 * e.oN1 + n2 * e.oN2s + (int64_t)wo0 + quarter * 32;
  const int row_lim = c.Wo - wo0 - quarter * 32;  // valid positions of this warp: r < row_lim
  const int rq = 4 * (lane & 7);
  const bool full4 = rq + 4 <= row_lim;
  const bool glu = e.mode == EPI_CONV && e.act >= 2;
  float gmu = 0.f, grs = 0.f;
  if (e.mode == EPI_CONV && e.act == 3) {
    gmu = e.gn_mean[n];
    grs = e.gn_rstd[n];
  }
  const int ncols = glu ? e.glu_half : BN;
  const int per = ncols >= 32 ? ncols / 2 : (half == 0 ? ncols : 0);
  const int cbeg = ncols >= 32 ? half * per : 0;
  const int obase = glu ? nt * e.glu_half : nt * BN;
  for (int c0 = cbeg; c0 < cbeg + per; c0 += 16) {
    float va[16];
    tmem_ld16(trow + c0, va);
    // per-column constants: lane i < 16 loads column i's, shuffles hand them out
    const int li = lane & 15;
    const int colx = obase + c0 + li;
    if (glu) {
      float vb[16];
      tmem_ld16(trow + e.glu_half + c0, vb);
      const bool okc = colx < e.O;
      const float ba = okc && e.bias ? e.bias[colx] : 0.f;
      const float bb = okc && e.bias ? e.bias[e.O + colx] : 0.f;
      float wa = 1.f, wb = 1.f, za = 0.f, zb = 0.f;
      if (e.act == 3 && okc) {
        wa = e.gn_w[colx] * grs;
        wb = e.gn_w[e.O + colx] * grs;
        za = e.gn_b[colx];
        zb = e.gn_b[e.O + colx];
      }
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const float bai = __shfl_sync(0xffffffffu, ba, i);
        const float bbi = __shfl_sync(0xffffffffu, bb, i);
        float a = va[i] + bai, b = vb[i] + bbi;
        if (e.act == 3) {
          a = (a - gmu) * __shfl_sync(0xffffffffu, wa, i) + __shfl_sync(0xffffffffu, za, i);
          b = (b - gmu) * __shfl_sync(0xffffffffu, wb, i) + __shfl_sync(0xffffffffu, zb, i);
        }
        wst[i * 32 + lane] = obase + c0 + i < e.O ? a * sigmoid_fast(b) : 0.f;
      }
    } else {
      const int ox = e.mode == EPI_CONVTR ? colx % e.O : colx;
      const float bx = (e.bias && ox < e.O) ? e.bias[ox] : 0.f;
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) {
        float val = va[i] + __shfl_sync(0xffffffffu, bx, i);
        if (e.act == 1) val = gelu_f(val);
        wst[i * 32 + lane] = val;
      }
    }
    __syncwarp();
#pragma unroll
    for (int p = 0; p < 4; p++) {
      const int cc = (lane >> 3) + 4 * p;
      const int col = obase + c0 + cc;
      int64_t off;
      if (e.mode == EPI_CONVTR) {
        const int s = col / e.O, o = col - s * e.O;
        const int t = ho * e.stride + s - e.crop;
        if (s >= e.stride || t < 0 || t >= e.out_len) continue;
        off = base + (int64_t)o * e.oC + (int64_t)t * e.oH;
      } else {
        if (col >= e.O) continue;
        off = base + (int64_t)col * e.oC + (int64_t)ho * e.oH;
      }
      const float4 v4 = *(const float4 *)(wst + cc * 32 + rq);
      float vv[4] = {v4.x, v4.y, v4.z, v4.w};
      const int64_t a = off + rq;
      const uintptr_t al = (uintptr_t)(e.y + a) | (e.res ? (uintptr_t)(e.res + a) : 0);
      if (full4 && (al & 15) == 0) {
        if (e.res) {
          const float4 rr = *(const float4 *)(e.res + a);
          const float sc = e.scale[col];
          vv[0] = rr.x + sc * vv[0];
          vv[1] = rr.y + sc * vv[1];
          vv[2] = rr.z + sc * vv[2];
          vv[3] = rr.w + sc * vv[3];
        }
        *(float4 *)(e.y + a) = make_float4(vv[0], vv[1], vv[2], vv[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          if (rq + i >= row_lim) continue;
          float val = vv[i];
          if (e.res) val = e.res[a + i] + e.scale[col] * val;
          e.y[a + i] = val;
        }
      }
    }
    __syncwarp();
  }
}

template <int BN, bool X2>
__global__ void __launch_bounds__(kCtThreads, 1)
    k_conv_tma(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmX2,
               const __grid_constant__ CUtensorMap tmB, const ConvTma c, const Epi e) {
  using Cfg = CtCfg<BN, X2>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int stages = c.stages, xstages = c.xstages;
  const uint32_t xbytes = (uint32_t)c.bw * 64 * 4;  // one box (a multiple of 1024 bytes)
  const uint32_t xstage = xbytes * (X2 ? 2 : 1);
  // [operand stages: A tile | B tile][box stages: x box | x2 box][epilogue buffers]
  uint8_t *sAB = smem;
  uint8_t *sX = smem + (size_t)stages * Cfg::kABStage;
  float *stg = (float *)(sX + (size_t)xstages * xstage);  // 8 warps x [16][32] fp32
  uint64_t *xfull = (uint64_t *)(stg + 8 * kCtEpiCW * 32);
  uint64_t *xempty = xfull + xstages;
  uint64_t *bfull = xempty + xstages;
  uint64_t *afull = bfull + stages;
  uint64_t *empty = afull + stages;
  uint64_t *acc_full = empty + stages;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *fin = acc_empty + 2;
  uint32_t *tslot = (uint32_t *)(fin + 1);

  __shared__ uint32_t s_abort;
  if (threadIdx.x == 0) s_abort = fault_pending() ? 1u : 0u;
  __syncthreads();
  if (s_abort) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles_total = c.lines * c.tpl * c.ntiles;
  const int ngroups = c.KH * c.ncb;  // boxes per tile

  if (threadIdx.x == 0) {
    for (int i = 0; i < xstages; i++) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], 8);
    }
    for (int i = 0; i < stages; i++) {
      mbar_init(&bfull[i], 1);
      mbar_init(&afull[i], 8);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    mbar_init(fin, 1);
    fence_mbar_init();
  }
  if (warp == kCtMmaWarp) {
    tmem_alloc(tslot, (uint32_t)Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == kCtTmaWarp) {
    // ---- TMA producer: per (kh, channel block) one box, then the KW B tiles
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      if (X2) tma_prefetch_desc(&tmX2);
      tma_prefetch_desc(&tmB);
      uint32_t it = 0, xi = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < ntiles_total; tile += gridDim.x) {
        int64_t line;
        int wo0, nt;
        ct_tile(c, tile, line, wo0, nt);
        const int64_t n = line / c.Ho;
        const int ho = (int)(line - n * c.Ho);
        const int n1 = (int)(n / c.N2), n2 = (int)(n - (int64_t)n1 * c.N2);
        const int w_al = (wo0 - c.PW) & ~3;  // 16-byte aligned box start
        for (int grp = 0; ok && grp < ngroups; grp++, xi++) {
          const int kh = grp / c.ncb, cb = grp - kh * c.ncb;
          const int xs = (int)(xi % (uint32_t)xstages);
          if (!mbar_wait(&xempty[xs], ((xi / (uint32_t)xstages) & 1u) ^ 1u, kFaultEmpty)) {
            ok = false;
            break;
          }
          const int h = ho * c.SH - c.PH + kh * c.DH;
          uint8_t *xb = sX + (size_t)xs * xstage;
          mbar_expect_tx(&xfull[xs], xstage);
          tma_load_5d(xb, &tmX, &xfull[xs], w_al, h, cb * 64, n2, n1);
          if (X2) tma_load_5d(xb + xbytes, &tmX2, &xfull[xs], w_al, h, cb * 64, n2, n1);
          for (int kw = 0; kw < c.KW; kw++, it++) {
            const int st = (int)(it % (uint32_t)stages);
            if (!mbar_wait(&empty[st], ((it / (uint32_t)stages) & 1u) ^ 1u, kFaultEmpty)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&bfull[st], Cfg::kBBytes);
            tma_load_3d(sAB + (size_t)st * Cfg::kABStage + kATileBytes, &tmB, &bfull[st],
                        (grp * c.KW + kw) * kBK, nt * BN, 0);
          }
        }
      }
    }
  } else if (warp == kCtMmaWarp) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(kBM, BN);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < ntiles_total; tile += gridDim.x, local++) {
        const uint32_t buf = local & 1u, use = local >> 1;
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, kFaultDone)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * (uint32_t)Cfg::kAccCols;
        for (int kb = 0; kb < c.nkb; kb++, it++) {
          const int st = (int)(it % (uint32_t)stages);
          const uint32_t ph = (it / (uint32_t)stages) & 1u;
          if (!mbar_wait(&afull[st], ph, kFaultFull) || !mbar_wait(&bfull[st], ph, kFaultFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t *sb = sAB + (size_t)st * Cfg::kABStage;
          const uint64_t ad = sw128_desc(smem_u32(sb));
          const uint64_t bd = sw128_desc(smem_u32(sb + kATileBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; k++)
            umma_f16(d, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      umma_commit(fin);
      mbar_wait(fin, 0, kFaultDone);
    }
  } else if (warp >= 8) {
    // ---- converters: warp w = 8 + (half << 2) + q builds rows 32q..32q+31 (one output
    // position per thread) and channels 32 half..32 half+31 of each A tile
    const int cw = warp - 8;
    const int r = (cw & 3) * 32 + lane, ch0 = (cw >> 2) * 32;
    uint32_t it = 0, xi = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles_total; tile += gridDim.x) {
      int64_t line;
      int wo0, nt;
      ct_tile(c, tile, line, wo0, nt);
      const int sh0 = (wo0 - c.PW) - ((wo0 - c.PW) & ~3);
      for (int grp = 0; ok && grp < ngroups; grp++, xi++) {
        const int xs = (int)(xi % (uint32_t)xstages);
        if (!mbar_wait(&xfull[xs], (xi / (uint32_t)xstages) & 1u, kFaultFull)) {
          ok = false;
          break;
        }
        const float *xb = (const float *)(sX + (size_t)xs * xstage);
        for (int kw = 0; kw < c.KW; kw++, it++) {
          const int st = (int)(it % (uint32_t)stages);
          if (!mbar_wait(&empty[st], ((it / (uint32_t)stages) & 1u) ^ 1u, kFaultEmpty)) {
            ok = false;
            break;
          }
          const float *xs_r = xb + (size_t)ch0 * c.bw + r + sh0 + kw * c.DW;
          const uint32_t a_base = smem_u32(sAB + (size_t)st * Cfg::kABStage);
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; i++) {
            v[i] = xs_r[i * c.bw];
            if (X2) v[i] += xs_r[i * c.bw + 64 * c.bw];
          }
#pragma unroll
          for (int cc = 0; cc < 4; cc++)
            st_shared_v4(a_base + sw128_off(r, (ch0 >> 3) + cc), pack_h2(v[8 * cc], v[8 * cc + 1]),
                         pack_h2(v[8 * cc + 2], v[8 * cc + 3]),
                         pack_h2(v[8 * cc + 4], v[8 * cc + 5]),
                         pack_h2(v[8 * cc + 6], v[8 * cc + 7]));
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[st]);
        }
        // every A tile of this box is built: the box may be refilled
        __syncwarp();
        if (lane == 0) mbar_arrive(&xempty[xs]);
      }
    }
  } else {
    // ---- epilogue warps 0-7
    float *wst = stg + warp * (kCtEpiCW * 32);
    uint32_t local = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles_total; tile += gridDim.x, local++) {
      int64_t line;
      int wo0, nt;
      ct_tile(c, tile, line, wo0, nt);
      const uint32_t buf = local & 1u, use = local >> 1;
      if (!warp_all(mbar_wait(&acc_full[buf], use & 1u, kFaultDone))) break;
      tc_fence_after();
      ct_epilogue<BN>(c, e, tmem + buf * (uint32_t)Cfg::kAccCols, warp, lane, line, wo0, nt,
                      wst);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kCtMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------- fp16 channels-last conv
// Implicit-GEMM convolution whose A operand is an fp16 channels-last activation
// [images][H][W][C] written by the producing layer.  A tile is 128 consecutive output
// positions of one output line (n, ho); K blocks are (kh, 64-channel block, kw) and each
// is ONE TMA box of 64 channels x 128 positions, which lands in shared memory exactly as
// the K-major SWIZZLE_128B UMMA operand: the tap's position offset is the box coordinate,
// positions and channels outside the tensor read as zero (the zero padding), a stride of 4
// along W is a 5-D view (C, 4, W/4, H, images) of the same tensor.  No thread touches the
// operand: a TMA warp streams A and B tiles into a shared-memory ring, one thread issues
// tcgen05.mma into one of two TMEM accumulators, and 4 epilogue warps drain the other
// (bias / GELU / GLU / GroupNorm-GLU / transposed-conv phase scatter, fp32 NCHW output
// and/or the fp16 channels-last copy for the next conv).  Two CTAs per SM for N tiles up
// to 128 columns.
struct ConvH {
  int KH, KW, SH, SW, PH, PW, DH, DW;
  int Ho, Wo;
  int ncb;        // 64-channel blocks
  int64_t lines;  // output lines (images * Ho)
  int tpl;        // tiles of 128 positions per line
  int N, nkb, ntiles, stages;
  int kst_last;   // MMA K steps (16 channels each) of the last 64-channel block: the rest
                  // of that block is the tensor's zero fill, and its products are skipped
  int blocked;    // 1: each CTA takes one contiguous range of tiles (row statistics over
                  // few rows: a CTA's tiles then mostly share their row), else cyclically
};

constexpr int kChEpiWarps = 8;  // warp & 3: TMEM lane quarter, warp >> 2: column half
constexpr int kChTmaWarp = kChEpiWarps, kChMmaWarp = kChEpiWarps + 1;
constexpr int kChThreads = 32 * (kChEpiWarps + 2);

template <int BN>
struct ChCfg {
  static constexpr uint32_t kStage = kATileBytes + BN * 128;  // a multiple of 1024
  static constexpr int kAccCols = BN < 32 ? 32 : BN;
  // two accumulators, allocated as a power of two columns (96-column tiles take 256)
  static constexpr int kTmemCols = 2 * kAccCols <= 64 ? 64 : 2 * kAccCols <= 128 ? 128 : 256;
};

static __device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map,
                                                   uint64_t *bar, int c0, int c1, int c2,
                                                   int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// tile -> (line, first position, N tile), N tiles fastest (tile counts fit in 31 bits)
static __device__ __forceinline__ void ch_tile(const ConvH &c, int64_t tile, int64_t &line,
                                               int &wo0, int &nt) {
  const int t = (int)tile;
  const int rest = t / c.ntiles;
  nt = t - rest * c.ntiles;
  const int ln = rest / c.tpl;
  line = ln;
  wo0 = (rest - ln * c.tpl) * kBM;
}

// Epilogue of one line tile by 4 warps (warp w: rows 32w..32w+31, every column), 16
// columns per step.  Values go (1) from registers to the fp16 channels-last copy, 16
// consecutive channels of a position per thread, and (2) through the warp's [16][32]
// transpose buffer to the fp32 NCHW output, 4 consecutive positions per 16-byte store.
// Transposed-conv columns are (phase s, channel o), channels fastest; (s, o) of the
// chunk start advance incrementally (no divisions in the loop).
// e.row_stats: add a warp's share of an image's output sum and sum of squares (the
// GroupNorm(1) statistics of a DConv hidden row, Ho = 1: image = row), fp64 atomics
static __device__ __forceinline__ void row_stats_add(const Epi &e, int64_t n, int lane,
                                                     double s, double q) {
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  if (lane == 0 && q > 0.0) {
    atomicAdd(&e.row_stats[2 * n], s);
    atomicAdd(&e.row_stats[2 * n + 1], q);
  }
}

template <int BN>
static __device__ __forceinline__ void ch_epilogue(const ConvH &c, const Epi &e, uint32_t tacc,
                                                   int warp, int lane, int64_t line, int wo0,
                                                   int nt, float *wst, double &rsum,
                                                   double &rsq) {
  const int quarter = warp & 3, half = warp >> 2;
  const uint32_t trow = tacc + ((uint32_t)(quarter * 32) << 16);
  const int ln = (int)line;
  const int n = ln / c.Ho;
  const int ho = ln - n * c.Ho;
  const int n1 = n / e.oN2, n2 = n - n1 * e.oN2;
  const int64_t base = (int64_t)n1 * e.oN1 + (int64_t)n2 * e.oN2s;
  const int r = quarter * 32 + lane;
  const int row_lim = c.Wo - wo0;  // tile rows r < row_lim are outputs
  const bool rv = r < row_lim;
  const int q = wo0 + r;           // output position along W (conv, conv_tr along H) or q
  const bool convtr = e.mode == EPI_CONVTR;
  const bool glu = !convtr && e.act >= 2;
  const bool gelu = e.act == 1;
  const int O = e.O;
  float gmu = 0.f, grs = 0.f;
  if (glu && e.act == 3) {
    gmu = e.gn_mean[n];
    grs = e.gn_rstd[n];
  }
  const int ncols = glu ? e.glu_half : BN;
  // the two warps of a lane quarter split the 16-column chunks (the first takes the odd one)
  const int nch = ncols >> 4, h0 = (nch + 1) >> 1;
  const int per = 16 * (half == 0 ? h0 : nch - h0);
  const int cbeg = half == 0 ? 0 : 16 * h0;
  const int obase = (glu ? nt * e.glu_half : nt * BN) + cbeg;
  const int ncol_total = convtr ? O * e.stride : O;
  const int li = lane & 15;
  // transposed conv: phase and channel of the chunk's first column
  int s0 = convtr ? obase / O : 0;
  int o0 = convtr ? obase - s0 * O : obase;
  const bool o16 = O % 16 == 0;  // every chunk then lies in one phase
  const int rq = 4 * (lane & 7);
  const int rl = quarter * 32 + rq;  // first of this lane's 4 rows in the NCHW pass
  for (int c0 = 0; c0 < per; c0 += 16) {
    const int col0 = obase + c0;
    if (col0 >= ncol_total) break;
    float va[16];
    tmem_ld16(trow + cbeg + c0, va);
    // output coordinates of this lane's row for the chunk (conv: (ho, q))
    int h = ho, w = q;
    bool tok = true;
    if (convtr) {
      const int t = (e.axis_h ? ho : q) * e.stride + s0 - e.crop;
      tok = t >= 0 && t < e.out_len;
      if (e.axis_h) {
        h = t;
      } else {
        h = 0;
        w = t;
      }
    }
    const bool cl_fast = (!convtr || o16) && o0 + 16 <= O;  // 16 channels of one position
    // skip-connection (or residual) values for the fp16 copy, loaded before the
    // accumulator wait
    float sk[16];
    const bool want_h = e.yh && rv && tok && cl_fast;
    const float *skp = e.hskip ? e.hskip : e.res;
    if (want_h && skp) {
      const float *sp = skp + base + (int64_t)o0 * e.oC + (int64_t)h * e.oH + w;
#pragma unroll
      for (int i = 0; i < 16; i++) sk[i] = sp[(int64_t)i * e.oC];
    } else {
#pragma unroll
      for (int i = 0; i < 16; i++) sk[i] = 0.f;
    }
    // per-column constants: lane i < 16 loads column i's, shuffles hand them out
    const int oxl = o0 + li;  // channel of column li when the chunk lies in one phase
    int ox = oxl;
    if (convtr && !o16) ox = (col0 + li) % O;
    const bool okc = convtr ? col0 + li < ncol_total : oxl < O;
    float val[16];
    if (glu) {
      float vb[16];
      tmem_ld16(trow + e.glu_half + cbeg + c0, vb);
      const float ba = okc && e.bias ? e.bias[oxl] : 0.f;
      const float bb = okc && e.bias ? e.bias[O + oxl] : 0.f;
      float wa = 1.f, wb = 1.f, za = 0.f, zb = 0.f;
      if (e.act == 3 && okc) {
        wa = e.gn_w[oxl] * grs;
        wb = e.gn_w[O + oxl] * grs;
        za = e.gn_b[oxl];
        zb = e.gn_b[O + oxl];
      }
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) {
        float a = va[i] + __shfl_sync(0xffffffffu, ba, i);
        float b = vb[i] + __shfl_sync(0xffffffffu, bb, i);
        if (e.act == 3) {
          a = (a - gmu) * __shfl_sync(0xffffffffu, wa, i) + __shfl_sync(0xffffffffu, za, i);
          b = (b - gmu) * __shfl_sync(0xffffffffu, wb, i) + __shfl_sync(0xffffffffu, zb, i);
        }
        val[i] = a * sigmoid_fast(b);
      }
    } else {
      const float bx = (e.bias && okc) ? e.bias[ox] : 0.f;
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) {
        float v = va[i] + __shfl_sync(0xffffffffu, bx, i);
        if (gelu) v = gelu_f(v);
        val[i] = v;
      }
    }
    if (e.emb) {
      const float ex = okc ? e.emb_alpha * e.emb[(int64_t)ho * e.emb_ld + oxl] : 0.f;
#pragma unroll
      for (int i = 0; i < 16; i++) val[i] += __shfl_sync(0xffffffffu, ex, i);
    }
    if (e.row_stats && rv) {
      // (e.row_stats: this lane's sum and sum of squares of the row's outputs; the chunk's
      // 16 in fp32, the running totals in fp64)
      float s16 = 0.f, q16 = 0.f;
#pragma unroll
      for (int i = 0; i < 16; i++) {
        if (col0 + i < ncol_total) {
          s16 += val[i];
          q16 = fmaf(val[i], val[i], q16);
        }
      }
      rsum += (double)s16;
      rsq += (double)q16;
    }
    // ---- (1) fp16 channels-last copy: value + skip, or res + scale[o] * value
    float mul[16];
    if (e.res && !e.hskip && e.yh) {
      // (uniform branch: every lane takes part in the shuffles)
      const float scx = okc ? e.scale[oxl] : 0.f;
#pragma unroll
      for (int i = 0; i < 16; i++) mul[i] = __shfl_sync(0xffffffffu, scx, i);
    } else {
#pragma unroll
      for (int i = 0; i < 16; i++) mul[i] = 1.f;
    }
    if (want_h) {
      float hv[16];
#pragma unroll
      for (int i = 0; i < 16; i++) hv[i] = fmaf(val[i], mul[i], sk[i]);
      uint16_t *dst = e.yh + (((int64_t)n * e.yhH + h) * e.yhW + w) * e.yhC + o0;
      uint4 *d4 = (uint4 *)dst;
      d4[0] = make_uint4(pack_h2(hv[0], hv[1]), pack_h2(hv[2], hv[3]), pack_h2(hv[4], hv[5]),
                         pack_h2(hv[6], hv[7]));
      d4[1] = make_uint4(pack_h2(hv[8], hv[9]), pack_h2(hv[10], hv[11]),
                         pack_h2(hv[12], hv[13]), pack_h2(hv[14], hv[15]));
    } else if (e.yh && rv) {
      // partial chunk (channel tail, or a transposed-conv chunk across two phases)
      for (int i = 0; i < 16; i++) {
        const int col = col0 + i;
        if (col >= ncol_total) break;
        int ss = s0, o = o0 + i;
        if (convtr) {
          ss = col / O;
          o = col - ss * O;
        } else if (o >= O) {
          break;
        }
        int hh = ho, ww = q;
        if (convtr) {
          const int t = (e.axis_h ? ho : q) * e.stride + ss - e.crop;
          if (t < 0 || t >= e.out_len) continue;
          hh = e.axis_h ? t : 0;
          ww = e.axis_h ? q : t;
        }
        float v = val[i];
        const int64_t so = base + (int64_t)o * e.oC + (int64_t)hh * e.oH + ww;
        if (e.hskip) v += e.hskip[so];
        else if (e.res) v = e.res[so] + e.scale[o] * v;
        e.yh[(((int64_t)n * e.yhH + hh) * e.yhW + ww) * e.yhC + o] = f2h_bits(v);
      }
    }
    // ---- (2) fp32 NCHW output through the transpose buffer, 8 columns at a time
    if (e.y) {
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
#pragma unroll
        for (int i = 0; i < 8; i++) wst[i * 32 + lane] = val[hh * 8 + i];
        __syncwarp();
#pragma unroll
        for (int p = 0; p < 2; p++) {
          const int cl = (lane >> 3) + 4 * p;
          const int cc = hh * 8 + cl;
          const int col = col0 + cc;
          if (col >= ncol_total) continue;
          // (phase, channel) of the column without a division when O >= 16
          int ss = s0, o = o0 + cc;
          if (convtr) {
            if (O >= 16) {
              if (o >= O) {
                o -= O;
                ss++;
              }
            } else {
              ss = col / O;
              o = col - ss * O;
            }
          }
          const float4 v4 = *(const float4 *)(wst + cl * 32 + rq);
          const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
          if (convtr && !e.axis_h) {
            // phase scatter along W: output t = S q + s - crop
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const int t = (wo0 + rl + i) * e.stride + ss - e.crop;
              if (rl + i < row_lim && t >= 0 && t < e.out_len)
                e.y[base + (int64_t)o * e.oC + (int64_t)ho * e.oH + t] = vv[i];
            }
            continue;
          }
          int64_t off;
          if (convtr) {
            const int t = ho * e.stride + ss - e.crop;
            if (t < 0 || t >= e.out_len) continue;
            off = base + (int64_t)o * e.oC + (int64_t)t * e.oH + wo0 + rl;
          } else {
            off = base + (int64_t)col * e.oC + (int64_t)ho * e.oH + wo0 + rl;
          }
          const uintptr_t al =
              (uintptr_t)(e.y + off) | (e.res ? (uintptr_t)(e.res + off) : 0);
          if (rl + 4 <= row_lim && (al & 15) == 0) {
            float4 o4 = make_float4(vv[0], vv[1], vv[2], vv[3]);
            if (e.res) {
              const float4 rr = *(const float4 *)(e.res + off);
              const float sc = e.scale[col];
              o4 = make_float4(rr.x + sc * vv[0], rr.y + sc * vv[1], rr.z + sc * vv[2],
                               rr.w + sc * vv[3]);
            }
            *(float4 *)(e.y + off) = o4;
          } else {
#pragma unroll
            for (int i = 0; i < 4; i++) {
              if (rl + i >= row_lim) continue;
              float v = vv[i];
              if (e.res) v = e.res[off + i] + e.scale[col] * v;
              e.y[off + i] = v;
            }
          }
        }
        __syncwarp();
      }
    }
    // next chunk's (phase, channel)
    if (convtr) {
      o0 += 16;
      while (o0 >= O) {
        o0 -= O;
        s0++;
      }
    } else {
      o0 += 16;
    }
  }
}

// Specialised epilogue for the common layer shapes: every 16-column chunk is full (output
// columns a multiple of 16), column constants come from 16-byte aligned arrays (a
// transposed conv's bias expanded per (phase, channel) column), and the activation (ACT: 0
// none, 1 GELU, 2 GLU, 3 GroupNorm + GLU + LayerScale residual) and the output geometry
// (CT: 0 conv, 1 transposed conv along H, 2 along W) are compile-time.  The output value
// y of a DConv residual layer (res + scale * value) is formed once and serves both the
// fp16 channels-last copy and the fp32 NCHW output.  NCHW rows go through the warp's
// transpose buffer as 16-byte stores when they are 16-byte aligned (e.y_al), else straight
// from registers (lanes are consecutive positions, so each column is one coalesced store).
template <int BN, int ACT, int CT>
static __device__ __forceinline__ void ch_epi_fast(const ConvH &c, const Epi &e, uint32_t tacc,
                                                   int warp, int lane, int64_t line, int wo0,
                                                   int nt, float *wst, double &rsum,
                                                   double &rsq) {
  constexpr bool GLU = ACT >= 2;
  const int quarter = warp & 3, half = warp >> 2;
  const uint32_t trow = tacc + ((uint32_t)(quarter * 32) << 16);
  const int ln = (int)line;
  const int n = ln / c.Ho;
  const int ho = ln - n * c.Ho;
  const int n1 = n / e.oN2, n2 = n - n1 * e.oN2;
  const int64_t base = (int64_t)n1 * e.oN1 + (int64_t)n2 * e.oN2s;
  const int r = quarter * 32 + lane;
  const int row_lim = c.Wo - wo0;
  const bool rv = r < row_lim;
  const int q = wo0 + r;
  const int O = e.O;
  const int ncols = GLU ? e.glu_half : BN;
  const int nch = ncols >> 4, h0 = (nch + 1) >> 1;  // chunks of the two column halves
  const int per = 16 * (half == 0 ? h0 : nch - h0);
  const int cbeg = half == 0 ? 0 : 16 * h0;
  const int obase = (GLU ? nt * e.glu_half : nt * BN) + cbeg;
  const int ncol_total = CT != 0 ? O * e.stride : O;
  float gmu = 0.f, grs = 0.f;
  if constexpr (ACT == 3) {
    gmu = e.gn_mean[n];
    grs = e.gn_rstd[n];
  }
  const int rq = 4 * (lane & 7);
  const int rl = quarter * 32 + rq;  // first of this lane's 4 rows in the staged NCHW pass
  int s0 = 0, o0 = obase;            // (phase, channel) of the chunk's first column
  if constexpr (CT != 0) {
    s0 = obase / O;
    o0 = obase - s0 * O;
  }
  const float *cb = CT != 0 ? e.bias_x : e.bias;
  if constexpr (CT == 2) {
    if (e.spec_z) {
      // the last frequency decoder run along its frequency axis (line = time frame ho,
      // lane = input bin q): the de-normalised spectrum, frame-major.  Warp half h takes the
      // channel pairs (re, im) of [h O/2, (h + 1) O/2); phases (0, 1), then (2, 3), give
      // bins 4 q - crop + (0, 1), (2, 3): one 16-byte store per pair and phase pair, the
      // lanes' stores filling each other's 32-byte sectors
      const int Oh = O / 2, ob = half * Oh;
      const float sd = sqrtf(e.spec_var[n]) + e.spec_eps, mu = e.spec_mean[n];
      const int64_t rs = (int64_t)e.spec_frames * e.spec_bins;
      float2 *zr = e.spec_z + (int64_t)n * e.spec_rows * rs + (int64_t)ho * e.spec_bins;
#pragma unroll 1
      for (int sp = 0; sp < 2; sp++) {
        float a0[16], a1[16], b0[16], b1[16];
        tmem_ld16(trow + (uint32_t)(2 * sp * O + ob), a0);
        tmem_ld16(trow + (uint32_t)((2 * sp + 1) * O + ob), a1);
#pragma unroll
        for (int i = 0; i < 16; i++) {  // (the bias has O * 4 columns: read only Oh of 16)
          b0[i] = i < Oh ? cb[2 * sp * O + ob + i] : 0.f;
          b1[i] = i < Oh ? cb[(2 * sp + 1) * O + ob + i] : 0.f;
        }
        tmem_wait_ld();
        const int f = q * e.stride + 2 * sp - e.crop;  // even: both bins in or both out
        if (rv && f >= 0 && f + 1 < e.out_len) {
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            if (i < Oh) {
              const float4 v4 = make_float4(fmaf(a0[i] + b0[i], sd, mu),
                                            fmaf(a0[i + 1] + b0[i + 1], sd, mu),
                                            fmaf(a1[i] + b1[i], sd, mu),
                                            fmaf(a1[i + 1] + b1[i + 1], sd, mu));
              *(float4 *)(zr + (int64_t)((ob + i) >> 1) * rs + f) = v4;
            }
          }
        }
      }
      return;
    }
  }
  for (int c0 = 0; c0 < per; c0 += 16) {
    const int col0 = obase + c0;
    if (col0 >= ncol_total) break;
    float va[16], vb[16];
    tmem_ld16(trow + cbeg + c0, va);
    if constexpr (GLU) tmem_ld16(trow + e.glu_half + cbeg + c0, vb);
    // this lane's output position for the chunk's phase
    int h = ho, w = q;
    bool tok = true;
    if constexpr (CT == 1) {
      h = ho * e.stride + s0 - e.crop;
      tok = h >= 0 && h < e.out_len;
    } else if constexpr (CT == 2) {
      h = 0;
      w = q * e.stride + s0 - e.crop;
      tok = w >= 0 && w < e.out_len;
    }
    // skip connection of a decoder (transposed convs), laid out like y
    float sk[16];
#pragma unroll
    for (int i = 0; i < 16; i++) sk[i] = 0.f;
    if constexpr (CT != 0) {
      if (e.hskip != nullptr && rv && tok) {
        const float *sp = e.hskip + base + (int64_t)o0 * e.oC + (int64_t)h * e.oH + w;
#pragma unroll
        for (int i = 0; i < 16; i++) sk[i] = sp[(int64_t)i * e.oC];
      }
    }
    float ka[16];
    if (cb) {
      ld_cols16(cb + col0, ka);
    } else {
#pragma unroll
      for (int i = 0; i < 16; i++) ka[i] = 0.f;
    }
    float v[16];
    if constexpr (ACT == 2) {
      float kb[16];
      if (cb) {
        ld_cols16(cb + O + col0, kb);
      } else {
#pragma unroll
        for (int i = 0; i < 16; i++) kb[i] = 0.f;
      }
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) v[i] = (va[i] + ka[i]) * sigmoid_fast(vb[i] + kb[i]);
    } else if constexpr (ACT == 3) {
      // GroupNorm of the pre-GLU value: ((acc + bias) - mean) * rstd * g + beta, one GLU
      // half at a time (register pressure)
      float g[16], z[16];
      ld_cols16(e.gn_w + col0, g);
      ld_cols16(e.gn_b + col0, z);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) va[i] = fmaf((va[i] + ka[i]) - gmu, g[i] * grs, z[i]);
      ld_cols16(cb + O + col0, ka);
      ld_cols16(e.gn_w + O + col0, g);
      ld_cols16(e.gn_b + O + col0, z);
#pragma unroll
      for (int i = 0; i < 16; i++)
        v[i] = va[i] * sigmoid_fast(fmaf((vb[i] + ka[i]) - gmu, g[i] * grs, z[i]));
      // the residual (y itself, read before this thread's rows are rewritten)
      if (rv) {
        const float *sp = e.res + base + (int64_t)col0 * e.oC + (int64_t)ho * e.oH + q;
#pragma unroll
        for (int i = 0; i < 16; i++) sk[i] = sp[(int64_t)i * e.oC];
      }
    } else {
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) {
        v[i] = va[i] + ka[i];
        if constexpr (ACT == 1) v[i] = gelu_f(v[i]);
      }
    }
    if constexpr (CT == 0 && ACT != 3) {
      if (e.emb) {
        float em[16];
        ld_cols16(e.emb + (int64_t)ho * e.emb_ld + col0, em);
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = fmaf(e.emb_alpha, em[i], v[i]);
      }
    }
    if constexpr (CT == 0 && ACT == 0) {
      if (e.row_stats && rv) {
        float s16 = 0.f, q16 = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) {
          s16 += v[i];
          q16 = fmaf(v[i], v[i], q16);
        }
        rsum += (double)s16;
        rsq += (double)q16;
      }
    }
    // output value: res + scale * value (ACT 3); the fp16 copy adds the skip
    if constexpr (ACT == 3) {
      float sc[16];
      ld_cols16(e.scale + col0, sc);
#pragma unroll
      for (int i = 0; i < 16; i++) v[i] = fmaf(sc[i], v[i], sk[i]);
    }
    if (e.yh && rv && tok) {
      float hv[16];
#pragma unroll
      for (int i = 0; i < 16; i++) hv[i] = ACT == 3 ? v[i] : v[i] + sk[i];
      uint4 *d4 = (uint4 *)(e.yh + (((int64_t)n * e.yhH + h) * e.yhW + w) * e.yhC + o0);
      d4[0] = make_uint4(pack_h2(hv[0], hv[1]), pack_h2(hv[2], hv[3]), pack_h2(hv[4], hv[5]),
                         pack_h2(hv[6], hv[7]));
      d4[1] = make_uint4(pack_h2(hv[8], hv[9]), pack_h2(hv[10], hv[11]),
                         pack_h2(hv[12], hv[13]), pack_h2(hv[14], hv[15]));
    }
    if (e.y) {
      if (CT != 2 && e.y_al) {
        // 8 columns at a time through the transpose buffer: lane = (column, 4 rows)
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
#pragma unroll
          for (int i = 0; i < 8; i++) wst[i * 32 + lane] = v[hh * 8 + i];
          __syncwarp();
#pragma unroll
          for (int p = 0; p < 2; p++) {
            const int cl = (lane >> 3) + 4 * p;
            const int cc = hh * 8 + cl;
            int64_t off;
            bool ok = true;
            if constexpr (CT == 0) {
              off = base + (int64_t)(col0 + cc) * e.oC + (int64_t)ho * e.oH + wo0 + rl;
            } else {
              int o = o0 + cc, ss = s0;
              if (o >= O) {
                o -= O;
                ss++;
              }
              const int t = ho * e.stride + ss - e.crop;
              ok = t >= 0 && t < e.out_len;
              off = base + (int64_t)o * e.oC + (int64_t)t * e.oH + wo0 + rl;
            }
            if (ok) {
              const float4 v4 = *(const float4 *)(wst + cl * 32 + rq);
              if (rl + 4 <= row_lim) {
                *(float4 *)(e.y + off) = v4;
              } else {
                const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
                  if (rl + i < row_lim) e.y[off + i] = vv[i];
              }
            }
          }
          __syncwarp();
        }
      } else if (rv) {
        // lanes are consecutive positions: one coalesced store per column
#pragma unroll
        for (int i = 0; i < 16; i++) {
          if constexpr (CT == 0) {
            e.y[base + (int64_t)(col0 + i) * e.oC + (int64_t)ho * e.oH + q] = v[i];
          } else {
            int o = o0 + i, ss = s0;
            if (o >= O) {
              o -= O;
              ss++;
            }
            if constexpr (CT == 1) {
              const int t = ho * e.stride + ss - e.crop;
              if (t >= 0 && t < e.out_len)
                e.y[base + (int64_t)o * e.oC + (int64_t)t * e.oH + q] = v[i];
            } else {
              const int t = q * e.stride + ss - e.crop;
              if (t >= 0 && t < e.out_len)
                e.y[base + (int64_t)o * e.oC + (int64_t)ho * e.oH + t] = v[i];
            }
          }
        }
      }
    }
    // next chunk's (phase, channel); O >= 16, so at most one wrap
    o0 += 16;
    if constexpr (CT != 0) {
      if (o0 >= O) {
        o0 -= O;
        s0++;
      }
    }
  }
}

template <int BN, int EK>
__global__ void __launch_bounds__(kChThreads, 2)
    k_conv_h(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
             const ConvH c, const Epi e) {
  using Cfg = ChCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int stages = c.stages;
  float *stg = (float *)(smem + (size_t)stages * Cfg::kStage);  // 8 warps x [8][32] fp32
  uint64_t *full = (uint64_t *)(stg + kChEpiWarps * 8 * 32);
  uint64_t *empty = full + stages;
  uint64_t *acc_full = empty + stages;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *fin = acc_empty + 2;
  uint32_t *tslot = (uint32_t *)(fin + 1);

  __shared__ uint32_t s_abort;
  if (threadIdx.x == 0) s_abort = fault_pending() ? 1u : 0u;
  __syncthreads();
  if (s_abort) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles_total = c.lines * c.tpl * c.ntiles;
  // this CTA's tiles: t_beg, t_beg + t_step, .. < t_end (the same sequence for every role)
  int64_t t_beg = blockIdx.x, t_end = ntiles_total, t_step = gridDim.x;
  if (c.blocked) {
    const int64_t per = (ntiles_total + gridDim.x - 1) / gridDim.x;
    t_beg = (int64_t)blockIdx.x * per;
    t_end = t_beg + per < ntiles_total ? t_beg + per : ntiles_total;
    t_step = 1;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kChEpiWarps);
    }
    mbar_init(fin, 1);
    fence_mbar_init();
  }
  if (warp == kChMmaWarp) {
    tmem_alloc(tslot, (uint32_t)Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == kChTmaWarp) {
    // ---- TMA producer: per K block one A box (64 channels x 128 positions) and a B tile
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int st = 0;       // ring stage and its phase parity, and the K block's (kh, cb, kw),
      uint32_t ph = 0;  // all kept incrementally (no division in the issue loop)
      bool ok = true;
      for (int64_t tile = t_beg; ok && tile < t_end; tile += t_step) {
        int64_t line;
        int wo0, nt;
        ch_tile(c, tile, line, wo0, nt);
        const int64_t n = line / c.Ho;
        const int ho = (int)(line - n * c.Ho);
        int kh = 0, cb = 0, kw = 0;
        for (int kb = 0; kb < c.nkb; kb++) {
          if (!mbar_wait(&empty[st], ph ^ 1u, kFaultEmpty)) {
            ok = false;
            break;
          }
          const int h = ho * c.SH - c.PH + kh * c.DH;
          const int d = kw * c.DW - c.PW;  // tap offset along W
          uint8_t *sb = smem + (size_t)st * Cfg::kStage;
          mbar_expect_tx(&full[st], Cfg::kStage);
          if (c.SW == 1) {
            tma_load_4d(sb, &tmA, &full[st], cb * 64, wo0 + d, h, (int)n);
          } else {
            // input position 4 (wo0 + r) + d = 4 (q0 + r) + phase
            const int phase = ((d % 4) + 4) % 4, q0 = wo0 + (d - phase) / 4;
            tma_load_5d(sb, &tmA, &full[st], cb * 64, phase, q0, h, (int)n);
          }
          tma_load_3d(sb + kATileBytes, &tmB, &full[st], kb * kBK, nt * BN, 0);
          // K blocks run (kh, cb, kw) with kw fastest
          if (++kw == c.KW) {
            kw = 0;
            if (++cb == c.ncb) {
              cb = 0;
              kh++;
            }
          }
          if (++st == stages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == kChMmaWarp) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(kBM, BN);
      uint32_t local = 0;
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int64_t tile = t_beg; ok && tile < t_end; tile += t_step, local++) {
        const uint32_t buf = local & 1u, use = local >> 1;
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, kFaultDone)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * (uint32_t)Cfg::kAccCols;
        int cb = 0, kw = 0;  // channel block and W tap of the K block (kw fastest)
        for (int kb = 0; kb < c.nkb; kb++) {
          if (!mbar_wait(&full[st], ph, kFaultFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t *sb = smem + (size_t)st * Cfg::kStage;
          const uint64_t ad = sw128_desc(smem_u32(sb));
          const uint64_t bd = sw128_desc(smem_u32(sb + kATileBytes));
          // the last channel block may hold fewer than 64 channels
          const int kst = cb == c.ncb - 1 ? c.kst_last : kBK / 16;
#pragma unroll
          for (int k = 0; k < kBK / 16; k++)
            if (k < kst) umma_f16(d, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[st]);
          if (++kw == c.KW) {
            kw = 0;
            if (++cb == c.ncb) cb = 0;
          }
          if (++st == stages) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      umma_commit(fin);
      mbar_wait(fin, 0, kFaultDone);
    }
  } else {
    // ---- epilogue warps 0-3
    float *wst = stg + warp * (8 * 32);
    uint32_t local = 0;
    // e.row_stats: this warp's running sums of its current row, added to the row's totals
    // when the row changes and at the end (few atomics per row)
    double rsum = 0.0, rsq = 0.0;
    int64_t rrow = -1;
    for (int64_t tile = t_beg; tile < t_end; tile += t_step, local++) {
      int64_t line;
      int wo0, nt;
      ch_tile(c, tile, line, wo0, nt);
      if (e.row_stats) {
        const int64_t rn = line / c.Ho;
        if (rn != rrow) {
          if (rrow >= 0) row_stats_add(e, rrow, lane, rsum, rsq);
          rsum = 0.0;
          rsq = 0.0;
          rrow = rn;
        }
      }
      const uint32_t buf = local & 1u, use = local >> 1;
      if (!warp_all(mbar_wait(&acc_full[buf], use & 1u, kFaultDone))) break;
      tc_fence_after();
      // EK 0: generic epilogue; else the specialised one for ACT = (EK - 1) % 4 and
      // output geometry CT = (EK - 1) / 4
      if constexpr (EK == 0)
        ch_epilogue<BN>(c, e, tmem + buf * (uint32_t)Cfg::kAccCols, warp, lane, line, wo0, nt,
                        wst, rsum, rsq);
      else
        ch_epi_fast<BN, (EK - 1) % 4, (EK - 1) / 4>(c, e,
                                                    tmem + buf * (uint32_t)Cfg::kAccCols, warp,
                                                    lane, line, wo0, nt, wst, rsum, rsq);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (e.row_stats && rrow >= 0) row_stats_add(e, rrow, lane, rsum, rsq);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kChMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------- CUDA-core kernel
// Same contract, one thread per (row, column) with rows fastest (coalesced gathers).
template <bool GATHER>
__global__ void k_simt(RowsA a, RowsA b, const Shape s, const Gather g, const Epi e,
                       int64_t ncols) {
  const int bz = blockIdx.y;
  const int64_t total = (int64_t)s.M * ncols;
  DCB_GRID_STRIDE(idx, total) {
    const int64_t n = idx / s.M, m = idx - n * s.M;
    const bool glu = e.mode == EPI_CONV && e.act >= 2;
    // B rows used: n, or the interleaved GLU pair of output channel n
    int64_t rb0 = n, rb1 = -1;
    if (glu) {
      const int hb = e.glu_half;
      rb0 = (n / hb) * 2 * hb + (n % hb);
      rb1 = rb0 + hb;
    }
    const uint16_t *B0 = b.p + (int64_t)bz * b.stride + rb0 * b.ld;
    const uint16_t *B1 = glu ? b.p + (int64_t)bz * b.stride + rb1 * b.ld : nullptr;
    float acc0 = 0.f, acc1 = 0.f;
    int64_t base = 0;
    int h0 = 0, w0 = 0;
    if (GATHER) {
      const int64_t hw = (int64_t)g.Ho * g.Wo;
      const int64_t nn = m / hw, rem = m - nn * hw;
      const int ho = (int)(rem / g.Wo), wo = (int)(rem - (int64_t)ho * g.Wo);
      const int64_t n1 = nn / g.N2, n2 = nn - n1 * g.N2;
      h0 = ho * g.SH - g.PH;
      w0 = wo * g.SW - g.PW;
      base = n1 * g.sN1 + n2 * g.sN2;
    }
    const uint16_t *Arow = GATHER ? nullptr : a.p + (int64_t)bz * a.stride + m * a.ld;
    for (int k = 0; k < s.K; k++) {
      float av;
      if (GATHER) {
        const int c = k % g.C, kk = k / g.C, kh = kk / g.KW, kw = kk - kh * g.KW;
        const int hh = h0 + kh * g.DH, ww = w0 + kw * g.DW;
        float xv = 0.f;
        if (hh >= 0 && hh < g.H && ww >= 0 && ww < g.W) {
          const int64_t o = base + (int64_t)c * g.sC + (int64_t)hh * g.sH + ww;
          xv = g.x[o] + (g.x2 ? g.x2[o] : 0.f);
        }
        av = h2f_bits(f2h_bits(xv));
      } else {
        av = h2f_bits(Arow[k]);
      }
      acc0 += av * h2f_bits(B0[k]);
      if (glu) acc1 += av * h2f_bits(B1[k]);
    }
    const RowInfo ri = decode_row(e, m);
    if (glu) {
      store_glu(e, n, ri, acc0, acc1, m / ((int64_t)e.Ho * e.Wo));
    } else {
      store_elem(e, s, bz, m, n, ri, acc0);
    }
  }
}

// ------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static bool get_encoder() {
  if (g_encode) return true;
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn) {
    fail("cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  return true;
}

// fp16 [batch][rows][inner] with row stride ld and batch stride bstride (elements)
static bool encode_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows,
                       uint64_t batch, uint64_t ld, uint64_t bstride, uint32_t box_rows) {
  if (!get_encoder()) return false;
  if (((uintptr_t)base & 15) || (ld * 2) % 16 || (batch > 1 && (bstride * 2) % 16)) return false;
  cuuint64_t dims[3] = {inner, rows, batch};
  cuuint64_t strides[2] = {ld * 2, (batch > 1 ? bstride : rows * ld) * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims,
                        strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static bool al16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// can the epilogue store 16 consecutive columns with vector instructions?
static bool vec_ok(const Epi &e, int64_t N) {
  if (N % 16) return false;
  switch (e.mode) {
    case EPI_ROWS_F32:
      return al16(e.out) && e.ldo % 4 == 0 && (!e.res || (al16(e.res) && e.ldr % 4 == 0));
    case EPI_ROWS_F16:
      return al16(e.out) && e.ldo % 8 == 0;
    case EPI_HEADS:
      for (int i = 0; i < 3; i++)
        if (e.sec_ptr[i] && !al16(e.sec_ptr[i])) return false;
      return e.hd % 16 == 0 && e.sec_cols % 16 == 0;
    default:
      return false;
  }
}

// N tile: the widest of 256 / 128 / 64 / 32 whose padding (tiles * bn - N) is smallest
// (a narrower tile only when it wastes fewer columns), then narrowed while the grid has
// fewer tiles than SMs
static int pick_bn(int64_t M, int64_t N, int64_t batch) {
  int bn = 32;
  while (bn < 256 && bn < N) bn *= 2;
  int64_t best = ((N + bn - 1) / bn) * bn - N;
  for (int c = bn / 2; c >= 64; c /= 2) {
    const int64_t waste = ((N + c - 1) / c) * c - N;
    if (waste < best) {
      best = waste;
      bn = c;
    }
  }
  const int64_t mt = (M + kBM - 1) / kBM;
  while (bn > 32 && mt * ((N + bn - 1) / bn) * batch < 148) bn /= 2;
  return bn;
}

int gather_bn(int64_t M, int64_t N, bool glu) {
  // at most 128 columns: a double-buffered accumulator, two CTAs per SM
  int bn = pick_bn(M, N, 1);
  if (bn > 128) bn = 128;
  if (glu && bn < 32) bn = 32;
  return bn;
}

// persistent CTAs of k_umma per SM: 2 (two fit), 1 while another stream's kernels share the
// SMs (the cross transformer's two branches), where leaving room for them measured faster
// than filling every SM with GEMM tiles
int g_umma_ctas_per_sm = 2;

static int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  DCB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    n[dev] = v;
  }
  return n[dev];
}

template <int BN, bool GATHER, int EK>
static void launch_umma(const CUtensorMap &ta, const CUtensorMap &tb, Shape s, const Gather &g,
                        const Epi &e, int64_t mtiles, int ntiles, int64_t batch) {
  using Cfg = UmmaCfg<BN, GATHER>;
  const size_t table = GATHER ? (size_t)s.nkb * kBK * sizeof(int2) : 0;
  const size_t stage_bytes = kATileBytes + (size_t)Cfg::kBTileBytes;
  const size_t fixed = 1024 + (size_t)Cfg::kStageFloats * 4 + 16 + table;
  // two persistent CTAs per SM: <= 111 KB of dynamic shared memory and <= 256 TMEM
  // columns each
  const size_t budget = 111 * 1024;  // + 1 KB static + 1 KB reserved, twice <= 228 KB
  int stages = budget > fixed + 8 * 24 ? (int)((budget - fixed - 8 * 24) / (stage_bytes + 16))
                                       : 0;
  if (stages > 8) stages = 8;
  if (stages < 2) stages = 2;
  s.stages = stages;
  const size_t smem = fixed + (size_t)stages * stage_bytes + (2 * (size_t)stages + 5) * 8;
  DCB_REQUIRE(smem <= 226 * 1024, "gemm: shared memory %zu exceeds the per-CTA limit", smem);
  static size_t attr = 0;  // dynamic shared memory opted in so far for this instantiation
  if (smem > attr) {
    DCB_CUDA(cudaFuncSetAttribute(k_umma<BN, GATHER, EK>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = smem;
  }
  DCB_REQUIRE(mtiles < (1ll << 31) && batch < (1ll << 31), "gemm: too many tiles");
  s.mtiles = (int)mtiles;
  s.ntiles = ntiles;
  s.batch = (int)batch;
  const int64_t tiles = mtiles * ntiles * batch;
  const int64_t slots = (int64_t)g_umma_ctas_per_sm * sm_count();
  const unsigned grid = (unsigned)(tiles < slots ? tiles : slots);
  k_umma<BN, GATHER, EK><<<grid, kThreads, smem, stream()>>>(ta, tb, s, g, e);
  DCB_LAUNCHED();
}

template <bool GATHER>
static void dispatch_umma(int bn, const CUtensorMap &ta, const CUtensorMap &tb, Shape s,
                          const Gather &g, const Epi &e, int64_t batch) {
  const int64_t mt = (s.M + kBM - 1) / kBM;
  const int ntl = (int)((s.N + bn - 1) / bn);
  if constexpr (!GATHER) {
    if (e.cvec) {
      switch (bn) {
        case 32: launch_umma<32, false, 1>(ta, tb, s, g, e, mt, ntl, batch); break;
        case 64: launch_umma<64, false, 1>(ta, tb, s, g, e, mt, ntl, batch); break;
        case 128: launch_umma<128, false, 1>(ta, tb, s, g, e, mt, ntl, batch); break;
        default: launch_umma<256, false, 1>(ta, tb, s, g, e, mt, ntl, batch); break;
      }
      return;
    }
  }
  switch (bn) {
    case 32: launch_umma<32, GATHER, 0>(ta, tb, s, g, e, mt, ntl, batch); break;
    case 64: launch_umma<64, GATHER, 0>(ta, tb, s, g, e, mt, ntl, batch); break;
    case 128: launch_umma<128, GATHER, 0>(ta, tb, s, g, e, mt, ntl, batch); break;
    default:
      if constexpr (GATHER) {
        DCB_REQUIRE(false, "conv: N tile %d is wider than the gather kernel's 128", bn);
      } else {
        launch_umma<256, GATHER, 0>(ta, tb, s, g, e, mt, ntl, batch);
      }
      break;
  }
}

template <bool GATHER>
static void launch_simt(RowsA a, RowsA b, Shape s, const Gather &g, const Epi &e, int64_t ncols,
                        int64_t batch) {
  DCB_REQUIRE(batch <= 65535, "gemm (CUDA-core path): batch %lld > 65535", (long long)batch);
  const int64_t total = (int64_t)s.M * ncols;
  dim3 grid(grid_for(total, 256, 148 * 64), (unsigned)batch);
  k_simt<GATHER><<<grid, 256, 0, stream()>>>(a, b, s, g, e, ncols);
  DCB_LAUNCHED();
}

void gemm_rows_launch(int64_t M, int64_t N, int64_t K, RowsA a, RowsA b, int64_t batch,
                      const Epi &e, Shape s, Gather g);

void gemm_rows(int64_t M, int64_t N, int64_t K, RowsA a, RowsA b, int64_t batch, const Epi &e) {
  if (M <= 0 || N <= 0 || batch <= 0) return;
  DCB_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm: extents too large");
  Shape s{};
  s.M = (int)M;
  s.N = (int)N;
  s.K = (int)K;
  s.nkb = (int)((K + kBK - 1) / kBK);
  s.a_shared = a.stride == 0;
  s.b_shared = b.stride == 0;
  Gather g{};
  {
    // algorithmic work of this call (unpadded extents) and its minimum bytes: the fp16
    // operands once and the output once at its precision (plus C's read when beta != 0,
    // part of the GEMM's definition); a fused residual's read is the design's extra traffic
    const double mnk = 2.0 * (double)M * (double)N * (double)K * (double)batch;
    double out_b = (double)M * N * batch * (e.mode == EPI_ROWS_F32 || e.mode == EPI_GEMM ? 4 : 2);
    if (e.beta != 0.f) out_b *= 2;
    const double in_b = 2.0 * ((double)M * K * (a.stride ? batch : 1) +
                               (double)N * K * (b.stride ? batch : 1));
    TraceScope ts(e.mode == EPI_GEMM ? TR_GEMM : TR_LINEAR, mnk, in_b + out_b, M, N, K);
    gemm_rows_launch(M, N, K, a, b, batch, e, s, g);
  }
}

// e.row_stats of a row-mode output the specialised epilogue did not cover: one warp per
// output row, fp32 over the row, fp64 atomics into its group's sums
__global__ void k_rows_group_sums(const float *__restrict__ out, int64_t ldo, int64_t M,
                                  int64_t N, int64_t grp, double *__restrict__ sums) {
  const int lane = threadIdx.x & 31;
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= M) return;
  float ls = 0.f, lq = 0.f;
  for (int64_t c = lane; c < N; c += 32) {
    const float v = out[r * ldo + c];
    ls += v;
    lq = fmaf(v, v, lq);
  }
  double s = ls, q = lq;
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  if (lane == 0) {
    double *st = sums + 2 * (kStatSlots * (r / grp) + blockIdx.x % kStatSlots);
    atomicAdd(&st[0], s);
    atomicAdd(&st[1], q);
  }
}

static void rows_group_sums(const Epi &e, int64_t M, int64_t N) {
  k_rows_group_sums<<<grid_for(M * 32, 256, 1 << 30), 256, 0, stream()>>>(
      (const float *)e.out, e.ldo, M, N, e.stat_rows, e.row_stats);
  DCB_LAUNCHED();
}

void gemm_rows_launch(int64_t M, int64_t N, int64_t K, RowsA a, RowsA b, int64_t batch,
                      const Epi &e, Shape s, Gather g) {
  DCB_REQUIRE(!e.row_stats || (e.mode == EPI_ROWS_F32 && e.stat_rows > 0 && batch == 1),
              "gemm: row-group statistics need a single fp32 row-mode output");
  if (!g_opt_simt && K > 0 && batch <= 65535) {
    int bn = pick_bn(M, N, batch);
    // at most 128 columns: the accumulator is then double-buffered in TMEM, so a tile's
    // epilogue overlaps the next tile's MMAs.  (Halving the tile for short GEMMs until every
    // persistent CTA had two tiles made the transformer's linears no faster alone and the
    // two-stream forward 0.9 % slower: the narrower tiles re-read A once per extra column
    // tile while the other branch's kernels share the SMs.)
    if (bn > 128) bn = 128;
    CUtensorMap ta, tb;
    const bool ok =
        encode_map(&ta, a.p, (uint64_t)K, (uint64_t)M, s.a_shared ? 1 : (uint64_t)batch,
                   (uint64_t)a.ld, (uint64_t)a.stride, kBM) &&
        encode_map(&tb, b.p, (uint64_t)K, (uint64_t)N, s.b_shared ? 1 : (uint64_t)batch,
                   (uint64_t)b.ld, (uint64_t)b.stride, (uint32_t)bn);
    if (ok) {
      Epi ev = e;
      ev.vec = vec_ok(e, N) ? 1 : 0;
      ev.cvec = ev.vec && !g_opt_generic_epi && (!e.bias || al16(e.bias)) &&
                (!e.res || (e.gamma && al16(e.gamma)))
                    ? 1
                    : 0;
      dispatch_umma<false>(bn, ta, tb, s, g, ev, batch);
      if (e.row_stats && !ev.cvec) rows_group_sums(e, M, N);
      return;
    }
  }
  launch_simt<false>(a, b, s, g, e, N, batch);
  if (e.row_stats) rows_group_sums(e, M, N);
}

// fp32 activation view (W, H, C, N2, N1) as a 5-D tensor map with bw x 1 x 64 x 1 x 1
// boxes; strides of extent-1 dimensions are irrelevant and set to the span below them
static bool encode_act5(CUtensorMap *map, const float *x, const Gather &g, int64_t n1_count,
                        int bw) {
  if (!get_encoder() || !x || ((uintptr_t)x & 15)) return false;
  const int64_t ext[5] = {g.W, g.H, g.C, g.N2, n1_count};
  const int64_t st[4] = {g.sH, g.sC, g.sN2, g.sN1};
  cuuint64_t dims[5], strides[4];
  for (int i = 0; i < 5; i++) {
    if (ext[i] <= 0 || ext[i] > (1ll << 31)) return false;
    dims[i] = (cuuint64_t)ext[i];
  }
  int64_t span = ((int64_t)g.W * 4 + 15) / 16 * 16;
  for (int i = 0; i < 4; i++) {
    int64_t b = st[i] * 4;
    if (ext[i + 1] == 1 || b == 0) b = span;
    if (b % 16 || b <= 0 || b >= (1ll << 40)) return false;
    strides[i] = (cuuint64_t)b;
    if (b * ext[i + 1] > span) span = b * ext[i + 1];
  }
  cuuint32_t box[5] = {(cuuint32_t)bw, 1, 64, 1, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float *>(x), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, bool X2>
static void launch_conv_tma(const CUtensorMap &tx, const CUtensorMap &tx2, const CUtensorMap &tb,
                            ConvTma c, const Epi &e) {
  using Cfg = CtCfg<BN, X2>;
  const size_t xstage = (size_t)c.bw * 64 * 4 * (X2 ? 2 : 1);
  const size_t budget = 226 * 1024;
  const size_t fixed = 1024 + (size_t)8 * kCtEpiCW * 32 * 4 + 5 * 8 + 16;
  auto need = [&](int xs, int st) {
    return fixed + (size_t)xs * (xstage + 16) + (size_t)st * (Cfg::kABStage + 24);
  };
  int xs = X2 ? 2 : 3, st = 6;
  while (st > 2 && need(xs, st) > budget) st--;
  if (need(xs, st) > budget) xs = 2;
  DCB_REQUIRE(need(xs, st) <= budget, "conv: TMA im2col stages do not fit in shared memory");
  c.xstages = xs;
  c.stages = st;
  const size_t smem = need(xs, st);
  static size_t attr = 0;
  if (smem > attr) {
    DCB_CUDA(cudaFuncSetAttribute(k_conv_tma<BN, X2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    attr = smem;
  }
  const int64_t tiles = c.lines * c.tpl * c.ntiles;
  const int64_t sms = sm_count();
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  k_conv_tma<BN, X2><<<grid, kCtThreads, smem, stream()>>>(tx, tx2, tb, c, e);
  DCB_LAUNCHED();
}

// fp16 channels-last activation as a TMA tensor map: 4-D (C, Wp, H, images), or with a
// stride of 4 along W the 5-D view (C, 4, Wp / 4, H, images); boxes of 64 channels x 128
// positions with the 128-byte swizzle of the UMMA operand
static bool encode_half(CUtensorMap *map, const HalfAct &x, bool w4) {
  if (!get_encoder() || !x.p || ((uintptr_t)x.p & 15) || x.C % 8 || x.Wp < x.W) return false;
  if (w4 && (x.Wp % 4 || x.sW || x.sH || x.sN)) return false;
  const uint64_t rowb = (uint64_t)x.C * 2;  // bytes per position
  // position strides along W, H and images (a strided view, else [images][H][Wp])
  const uint64_t sw = x.sW ? (uint64_t)x.sW : 1, sh = x.sH ? (uint64_t)x.sH : (uint64_t)x.Wp;
  const uint64_t sn = x.sN ? (uint64_t)x.sN : (uint64_t)x.Wp * x.H;
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5], es[5] = {1, 1, 1, 1, 1};
  int rank;
  if (!w4) {
    rank = 4;
    dims[0] = (cuuint64_t)x.C;
    dims[1] = (cuuint64_t)x.Wp;
    dims[2] = (cuuint64_t)x.H;
    dims[3] = (cuuint64_t)x.images;
    strides[0] = rowb * sw;
    strides[1] = rowb * sh;
    strides[2] = rowb * sn;
    box[0] = 64;
    box[1] = kBM;
    box[2] = 1;
    box[3] = 1;
  } else {
    rank = 5;
    dims[0] = (cuuint64_t)x.C;
    dims[1] = 4;
    dims[2] = (cuuint64_t)(x.Wp / 4);
    dims[3] = (cuuint64_t)x.H;
    dims[4] = (cuuint64_t)x.images;
    strides[0] = rowb;
    strides[1] = rowb * 4;
    strides[2] = rowb * x.Wp;
    strides[3] = rowb * x.Wp * x.H;
    box[0] = 64;
    box[1] = 1;
    box[2] = kBM;
    box[3] = 1;
    box[4] = 1;
  }
  for (int i = 0; i < rank - 1; i++)
    if (strides[i] % 16 || strides[i] >= (1ull << 40)) return false;
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<uint16_t *>(x.p), dims,
                  strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EK>
static void launch_conv_h_k(const CUtensorMap &ta, const CUtensorMap &tb, ConvH c,
                            const Epi &e) {
  using Cfg = ChCfg<BN>;
  // two CTAs per SM when the accumulators fit (<= 256 TMEM columns each)
  const bool two = Cfg::kTmemCols <= 256;
  const size_t budget = two ? 111 * 1024 : 226 * 1024;
  const size_t fixed = 1024 + (size_t)kChEpiWarps * 8 * 32 * 4 + 5 * 8 + 16;
  int stages = (int)((budget - fixed) / (Cfg::kStage + 16));
  if (stages > 8) stages = 8;
  DCB_REQUIRE(stages >= 2, "conv: stages do not fit in shared memory");
  c.stages = stages;
  const size_t smem = fixed + (size_t)stages * (Cfg::kStage + 16);
  static size_t attr = 0;
  if (smem > attr) {
    DCB_CUDA(cudaFuncSetAttribute(k_conv_h<BN, EK>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = smem;
  }
  const int64_t tiles = c.lines * c.tpl * c.ntiles;
  const int64_t slots = (two ? 2 : 1) * (int64_t)sm_count();
  const unsigned grid = (unsigned)(tiles < slots ? tiles : slots);
  k_conv_h<BN, EK><<<grid, kChThreads, smem, stream()>>>(ta, tb, c, e);
  DCB_LAUNCHED();
}

template <int BN>
static void launch_conv_h(const CUtensorMap &ta, const CUtensorMap &tb, ConvH c, const Epi &e,
                          int ek) {
  switch (ek) {
    case 1: launch_conv_h_k<BN, 1>(ta, tb, c, e); break;
    case 2: launch_conv_h_k<BN, 2>(ta, tb, c, e); break;
    case 3: launch_conv_h_k<BN, 3>(ta, tb, c, e); break;
    case 4: launch_conv_h_k<BN, 4>(ta, tb, c, e); break;
    case 5: launch_conv_h_k<BN, 5>(ta, tb, c, e); break;
    case 6: launch_conv_h_k<BN, 6>(ta, tb, c, e); break;
    case 9: launch_conv_h_k<BN, 9>(ta, tb, c, e); break;
    case 10: launch_conv_h_k<BN, 10>(ta, tb, c, e); break;
    default: launch_conv_h_k<BN, 0>(ta, tb, c, e); break;
  }
}

// Epilogue kind of a channels-last conv: 0 = the generic epilogue, else 1 + ACT + 4 * CT
// for the specialised one when its layout conditions hold (see ch_epi_fast); also sets
// e.y_al when the NCHW rows take 16-byte stores.
static int conv_epi_kind(Epi &e, int bn) {
  const bool tr = e.mode == EPI_CONVTR;
  const int act = e.act;
  const int O = e.O;
  e.y_al = 0;
  if (e.y && al16(e.y) && e.oC % 4 == 0 && e.oH % 4 == 0 && e.oN1 % 4 == 0 &&
      e.oN2s % 4 == 0)
    e.y_al = 1;
  if (tr) {
    if (act > 1 || e.res || O < 16 || (O * e.stride) % 16 != 0) return 0;
    if (e.spec_z) {
      // the spectrum epilogue: whole 16-byte bin pairs, and 16 TMEM columns from each
      // phase's channel half inside the accumulator
      if (e.axis_h || act != 0 || e.y || e.yh || e.hskip || e.stride != 4 || O % 8 != 0 ||
          O / 2 > 16 || 3 * O + O / 2 + 16 > bn || e.crop % 2 != 0 || e.spec_bins % 2 != 0 ||
          !e.bias_x || !al16(e.spec_z))
        return 0;
      return 1 + 0 + 4 * 2;
    }
    if (e.yh && O % 16 != 0) return 0;
    if (e.hskip && (!e.yh || O % 16 != 0)) return 0;  // skip rows are read 16 channels at a time
    if (e.bias && (!e.bias_x || !al16(e.bias_x))) return 0;
    if (e.emb) return 0;
    return 1 + act + 4 * (e.axis_h ? 1 : 2);
  }
  if (O % 16 != 0 || e.hskip) return 0;
  if (act >= 2 && (bn / 2) % 16 != 0) return 0;
  if (e.bias && !al16(e.bias)) return 0;
  if (e.emb && (act == 3 || !al16(e.emb) || e.emb_ld % 4 != 0)) return 0;
  if (act == 3) {
    if (!e.bias || !e.res || !e.scale || !e.gn_w || !e.gn_b || !al16(e.gn_w) ||
        !al16(e.gn_b) || !al16(e.scale))
      return 0;
  } else if (e.res) {
    return 0;
  }
  return 1 + act;
}

bool conv_half(const HalfAct &x, int KH, int KW, int SH, int SW, int PH, int PW, int DH, int DW,
               int Ho, int Wo, const uint16_t *wt, int64_t N, int64_t ldt, int ncb, const Epi &e,
               int bn_hint) {
  if (g_opt_simt || !wt || ncb <= 0 || (SW != 1 && SW != 4) || Ho <= 0 || Wo <= 0 || N <= 0)
    return false;
  if ((int64_t)KH * KW * ncb * kBK != ldt || (ncb - 1) * 64 >= x.C) return false;
  if (e.mode != EPI_CONV && e.mode != EPI_CONVTR) return false;
  if (e.mode == EPI_CONVTR && e.act >= 2) return false;
  const bool glu = e.mode == EPI_CONV && e.act >= 2;
  int bn = bn_hint ? bn_hint : pick_bn((int64_t)x.images * Ho * Wo, N, 1);
  if (glu && !bn_hint) return false;  // the GLU interleave fixes the N tile
  // at most 128 columns: two CTAs (8 epilogue warps) per SM drain the accumulators
  if (bn > 128) bn = 128;
  CUtensorMap ta, tb;
  if (!encode_half(&ta, x, SW == 4)) return false;
  if (!encode_map(&tb, wt, (uint64_t)ldt, (uint64_t)N, 1, (uint64_t)ldt, 0, (uint32_t)bn))
    return false;
  ConvH c{};
  c.KH = KH;
  c.KW = KW;
  c.SH = SH;
  c.SW = SW;
  c.PH = PH;
  c.PW = PW;
  c.DH = DH;
  c.DW = DW;
  c.Ho = Ho;
  c.Wo = Wo;
  c.ncb = ncb;
  c.lines = x.images * Ho;
  c.tpl = (Wo + kBM - 1) / kBM;
  c.N = (int)N;
  c.nkb = KH * KW * ncb;
  c.kst_last = (x.C - (ncb - 1) * 64 + 15) / 16;
  // row statistics over few long rows: contiguous tile ranges (each CTA then adds a row's
  // sums a few times instead of every CTA adding to every row); many rows keep the cyclic
  // order (neighbouring tiles run together, sharing their input halo in L2)
  c.blocked = e.row_stats != nullptr && x.images * Ho < 2LL * 2 * sm_count();
  if (c.kst_last > kBK / 16) c.kst_last = kBK / 16;
  c.ntiles = (int)((N + bn - 1) / bn);
  Epi e2 = e;
  if (glu) e2.glu_half = bn / 2;
  const int ek = g_opt_generic_epi ? 0 : conv_epi_kind(e2, bn);
  if (ek == 0 && e2.spec_z) return false;  // only the specialised epilogue writes it
  // row statistics: the generic and the plain (ACT 0) conv epilogues, one row per image
  if (e2.row_stats && (e.mode != EPI_CONV || ek > 1 || Ho != 1)) return false;
  {
    const int64_t M = x.images * Ho * Wo;
    const double n_alg = e.mode == EPI_CONVTR ? (double)e.O * e.stride : (glu ? 2.0 * e.O : e.O);
    const int Kt = KH * KW * x.C;
    // minimum bytes: the fp16 input and weights once and the output once at its precision
    // (fp32 when the fp32 tensor is written, else the fp16 copy); the extra fp16
    // channels-last copy and the decoder skip read are the design's traffic, not counted
    const double out_b =
        (double)M * n_alg / (glu ? 2 : 1) * (e.y || e.spec_z ? 4.0 : (e.yh ? 2.0 : 0.0));
    TraceScope ts(e.mode == EPI_CONVTR ? TR_CONVTR : TR_CONV, 2.0 * M * n_alg * Kt,
                  (double)x.images * x.H * x.W * x.C * 2.0 + n_alg * Kt * 2.0 + out_b, M,
                  (int64_t)n_alg, Kt);
    switch (bn) {
      case 32: launch_conv_h<32>(ta, tb, c, e2, ek); break;
      case 64: launch_conv_h<64>(ta, tb, c, e2, ek); break;
      case 96: launch_conv_h<96>(ta, tb, c, e2, ek); break;
      case 128: launch_conv_h<128>(ta, tb, c, e2, ek); break;
      default: launch_conv_h<256>(ta, tb, c, e2, ek); break;
    }
  }
  return true;
}

// TMA im2col path of gemm_gather: true when it launched
static bool conv_tma(const Gather &g, int64_t M, const uint16_t *wt, int64_t N, int64_t ldt,
                     int ncb, const Epi &e, int bn) {
  if (!wt || ncb <= 0 || g.SW != 1 || g.C < 32 || g.Wo < 64) return false;
  if (e.mode == EPI_CONVTR && !e.axis_h) return false;  // taps along W: no line tiles
  const int bw = (131 + (g.KW - 1) * g.DW + 3) / 4 * 4;
  if (bw > kCtBoxMax) return false;
  if ((int64_t)g.KH * g.KW * ncb * kBK != ldt) return false;
  const int64_t hw = (int64_t)g.Ho * g.Wo;
  if (hw <= 0 || M % hw) return false;
  const int64_t images = M / hw;
  if (images % g.N2) return false;
  const bool x2 = g.x2 != nullptr;
  if (x2 && bn > 128) bn = 128;
  CUtensorMap tx, tx2, tb;
  if (!encode_act5(&tx, g.x, g, images / g.N2, bw)) return false;
  if (x2 && !encode_act5(&tx2, g.x2, g, images / g.N2, bw)) return false;
  if (!encode_map(&tb, wt, (uint64_t)ldt, (uint64_t)N, 1, (uint64_t)ldt, 0, (uint32_t)bn))
    return false;
  ConvTma c{};
  c.KH = g.KH;
  c.KW = g.KW;
  c.SH = g.SH;
  c.PH = g.PH;
  c.DH = g.DH;
  c.PW = g.PW;
  c.DW = g.DW;
  c.Ho = g.Ho;
  c.Wo = g.Wo;
  c.ncb = ncb;
  c.lines = images * g.Ho;
  c.tpl = (g.Wo + kBM - 1) / kBM;
  c.N2 = g.N2;
  c.bw = bw;
  c.N = (int)N;
  c.nkb = g.KH * g.KW * ncb;
  c.ntiles = (int)((N + bn - 1) / bn);
  Epi e2 = e;
  if (e.mode == EPI_CONV && e.act >= 2) e2.glu_half = bn / 2;
  if (!x2) tx2 = tx;
  switch (bn) {
    case 32: x2 ? launch_conv_tma<32, true>(tx, tx2, tb, c, e2)
                : launch_conv_tma<32, false>(tx, tx2, tb, c, e2); break;
    case 64: x2 ? launch_conv_tma<64, true>(tx, tx2, tb, c, e2)
                : launch_conv_tma<64, false>(tx, tx2, tb, c, e2); break;
    case 128: x2 ? launch_conv_tma<128, true>(tx, tx2, tb, c, e2)
                 : launch_conv_tma<128, false>(tx, tx2, tb, c, e2); break;
    default: launch_conv_tma<256, false>(tx, tx2, tb, c, e2); break;
  }
  return true;
}

void gemm_gather(const Gather &g, int64_t M, const uint16_t *w, int64_t N, int64_t ldw,
                 const Epi &e, int bn_hint, const uint16_t *wt, int64_t ldt, int ncb) {
  if (M <= 0 || N <= 0) return;
  DCB_REQUIRE(M < (1ll << 31), "conv: too many output positions");
  Shape s{};
  s.M = (int)M;
  s.N = (int)N;
  s.K = g.K;
  s.nkb = (g.K + kBK - 1) / kBK;
  s.a_shared = 1;
  s.b_shared = 1;
  const bool glu = e.mode == EPI_CONV && e.act >= 2;
  const int bn = bn_hint ? bn_hint : gather_bn(M, N, glu);
  const double images = (double)M / ((double)g.Ho * g.Wo);
  const double n_alg = e.mode == EPI_CONVTR ? (double)e.O * e.stride : (glu ? 2.0 * e.O : e.O);
  const double out_elems = e.mode == EPI_CONVTR ? (double)M * e.O * e.stride : (double)M * e.O;
  // minimum bytes: the input once at the precision it is read in (fp32 here), the fp16
  // weights once and the fp32 output once (a second summed input and a fused residual are
  // the design's traffic)
  const double x_b = images * g.C * g.H * g.W * 4.0;
  TraceScope ts(e.mode == EPI_CONVTR ? TR_CONVTR : TR_CONV, 2.0 * M * n_alg * g.K,
                x_b + n_alg * g.K * 2.0 + out_elems * 4.0, M, (int64_t)n_alg, g.K);
  // a GLU N tile the tensor-core gather kernels do not take (96: the channels-last kernel's)
  const bool odd_tile = bn != 32 && bn != 64 && bn != 128;
  if (!g_opt_simt && !odd_tile) {
    // TMA im2col kernel (freq-branch convs); its N tile may be wider than the gather
    // kernel's, except for GLU convs whose weights are interleaved per N tile
    int bt = bn;
    if (!glu && !bn_hint) {
      bt = pick_bn(M, N, 1);
    }
    if (conv_tma(g, M, wt, N, ldt, ncb, e, bt)) return;
    CUtensorMap tb;
    // inner extent = the padded row length: padding columns are zero in every packed
    // weight, and a multiple-of-8 extent keeps the tensor map within TMA's 16-byte rules
    if (encode_map(&tb, w, (uint64_t)ldw, (uint64_t)N, 1, (uint64_t)ldw, 0, (uint32_t)bn)) {
      Epi e2 = e;
      if (glu) e2.glu_half = bn / 2;
      dispatch_umma<true>(bn, tb, tb, s, g, e2, 1);
      return;
    }
  }
  RowsA b{w, ldw, 0};
  Epi e2 = e;
  int64_t ncols = N;
  if (glu) {
    e2.glu_half = bn / 2;
    ncols = e.O;
  }
  launch_simt<true>(RowsA{nullptr, 0, 0}, b, s, g, e2, ncols, 1);
}

// -------- GLU weight interleave: rows [a | b] halves of O each -> per N tile of `bn`
// columns: bn/2 rows of the a-half followed by the matching bn/2 rows of the b-half.
__global__ void k_glu_interleave(const uint16_t *__restrict__ w, uint16_t *__restrict__ out,
                                 int O, int64_t kp, int hb, int ntiles) {
  int64_t total = (int64_t)ntiles * 2 * hb * kp;
  DCB_GRID_STRIDE(i, total) {
    int64_t row = i / kp, k = i - row * kp;
    int t = (int)(row / (2 * hb)), j = (int)(row % (2 * hb));
    int o = t * hb + (j < hb ? j : j - hb);
    uint16_t v = 0;
    if (o < O) v = w[((int64_t)(j < hb ? o : O + o)) * kp + k];
    out[i] = v;
  }
}

void glu_interleave(const uint16_t *w, uint16_t *out, int O, int64_t kp, int bn) {
  const int hb = bn / 2, ntiles = (O + hb - 1) / hb;
  int64_t total = (int64_t)ntiles * 2 * hb * kp;
  k_glu_interleave<<<grid_for(total, 256), 256, 0, stream()>>>(w, out, O, kp, hb, ntiles);
  DCB_LAUNCHED();
}

// -------- transposed-conv phase matrix: W_tr [O][KH][KW][C] (rows o*KH*KW + k, stride kp)
// -> B[(r, o)][(j', c)] = W[o][r + S (1 - j')][c], j' = 0 reads input q-1, j' = 1 input q.
__global__ void k_convtr_phase(const uint16_t *__restrict__ w, uint16_t *__restrict__ out,
                               int O, int C, int Ktaps, int S, int64_t kp, int64_t ldo) {
  int64_t total = (int64_t)O * S * ldo;
  DCB_GRID_STRIDE(i, total) {
    int64_t row = i / ldo, col = i - row * ldo;
    int r = (int)(row / O), o = (int)(row % O);  // rows (phase, channel), channels fastest
    uint16_t v = 0;
    if (col < 2 * C) {
      int jp = (int)(col / C), c = (int)(col % C);
      int tap = r + S * (1 - jp);
      if (tap < Ktaps) v = w[((int64_t)o * Ktaps + tap) * kp + c];
    }
    out[i] = v;
  }
}

void convtr_phase_matrix(const uint16_t *w, uint16_t *out, int O, int C, int Ktaps, int S,
                         int64_t kp, int64_t ldo) {
  int64_t total = (int64_t)O * S * ldo;
  k_convtr_phase<<<grid_for(total, 256), 256, 0, stream()>>>(w, out, O, C, Ktaps, S, kp, ldo);
  DCB_LAUNCHED();
}

}  // namespace dcb

using namespace dcb;

extern "C" {

void dk_gemm_half(int64_t M, int64_t N, int64_t K, float alpha, const dc_half *A, int64_t lda,
                  int64_t strideA, const dc_half *B, int64_t ldb, int64_t strideB, float beta,
                  float *C, int64_t ldc, int64_t strideC, int64_t batch) {
  if (M <= 0 || N <= 0 || batch <= 0) return;
  DCB_REQUIRE(K % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0,
              "dk_gemm_half: K, lda, ldb must be multiples of 8 (K=%lld lda=%lld ldb=%lld)",
              (long long)K, (long long)lda, (long long)ldb);
  Epi e;
  e.mode = EPI_GEMM;
  e.C = C;
  e.ldc = ldc;
  e.strideC = strideC;
  e.alpha = alpha;
  e.beta = beta;
  // Small M (conv weights as A, ops.c:55): put the long N side on the 128-row UMMA M
  // dimension and store the tile transposed.
  const bool swap = M < 128 && N > M;
  e.swapped = swap ? 1 : 0;
  for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
    const int64_t nb = batch - b0 < 65535 ? batch - b0 : 65535;
    RowsA a{A + b0 * strideA, lda, strideA}, b{B + b0 * strideB, ldb, strideB};
    Epi ec = e;
    ec.C = C + b0 * strideC;
    if (swap) {
      gemm_rows(N, M, K, b, a, nb, ec);
    } else {
      gemm_rows(M, N, K, a, b, nb, ec);
    }
  }
}

void dkx_conv2d(const float *x, int N, const DkConvGeom *g, const dc_half *weight, int O,
                const float *bias, int act, float *y) {
  Gather ga{};
  ga.x = x;
  ga.N2 = 1;
  ga.sN1 = (int64_t)g->C * g->H * g->W;
  ga.sN2 = 0;
  ga.sC = (int64_t)g->H * g->W;
  ga.sH = g->W;
  ga.C = g->C;
  ga.H = g->H;
  ga.W = g->W;
  ga.KH = g->KH;
  ga.KW = g->KW;
  ga.SH = g->SH;
  ga.SW = g->SW;
  ga.PH = g->PH;
  ga.PW = g->PW;
  ga.DH = g->DH;
  ga.DW = g->DW;
  ga.Ho = g->Ho;
  ga.Wo = g->Wo;
  ga.K = g->KH * g->KW * g->C;
  const int Oy = act == DKX_ACT_GLU ? O / 2 : O;
  Epi e;
  e.mode = EPI_CONV;
  e.bias = bias;
  e.act = act;
  e.y = y;
  e.oN2 = 1;
  e.oN1 = (int64_t)Oy * g->Ho * g->Wo;
  e.oC = (int64_t)g->Ho * g->Wo;
  e.oH = g->Wo;
  e.O = Oy;
  e.Ho = g->Ho;
  e.Wo = g->Wo;
  const int64_t M = (int64_t)N * g->Ho * g->Wo;
  if (act != DKX_ACT_GLU) {
    gemm_gather(ga, M, weight, O, g->Kp, e);
    return;
  }
  const int bn = gather_bn(M, O, true);
  const int hb = bn / 2, ntiles = (Oy + hb - 1) / hb;
  uint16_t *wi = nullptr;
  DCB_CUDA(cudaMallocAsync(&wi, (size_t)ntiles * bn * g->Kp * 2, stream()));
  glu_interleave(weight, wi, Oy, g->Kp, bn);
  gemm_gather(ga, M, wi, (int64_t)ntiles * bn, g->Kp, e, bn);
  DCB_CUDA(cudaFreeAsync(wi, stream()));
}

void dkx_conv_tr(const float *x, int N, int C, int H, int W, const dc_half *weight, int O,
                 int KH, int KW, int stride, const float *bias, int crop, int out_len,
                 int gelu, float *y) {
  const bool axis_h = KW == 1;
  const int Ktaps = axis_h ? KH : KW;
  DCB_REQUIRE((axis_h ? KW == 1 : KH == 1) && Ktaps == 2 * stride,
              "dkx_conv_tr: kernel must be 2*stride along one axis");
  const int64_t kp = (C + 7) / 8 * 8;  // loader rule: reduction over I padded to 8
  const int64_t K2 = 2 * (int64_t)C, ldo = (K2 + 7) / 8 * 8;
  uint16_t *ph = nullptr;
  DCB_CUDA(cudaMallocAsync(&ph, (size_t)O * stride * ldo * 2, stream()));
  convtr_phase_matrix(weight, ph, O, C, Ktaps, stride, kp, ldo);
  Gather ga{};
  ga.x = x;
  ga.N2 = 1;
  ga.sN1 = (int64_t)C * H * W;
  ga.sC = (int64_t)H * W;
  ga.sH = W;
  ga.C = C;
  ga.H = H;
  ga.W = W;
  ga.KH = axis_h ? 2 : 1;
  ga.KW = axis_h ? 1 : 2;
  ga.SH = ga.SW = 1;
  ga.PH = axis_h ? 1 : 0;
  ga.PW = axis_h ? 0 : 1;
  ga.DH = ga.DW = 1;
  ga.Ho = axis_h ? H + 1 : H;
  ga.Wo = axis_h ? W : W + 1;
  ga.K = 2 * C;
  const int Ho = axis_h ? out_len : H, Wo = axis_h ? W : out_len;
  Epi e;
  e.mode = EPI_CONVTR;
  e.bias = bias;
  e.act = gelu ? 1 : 0;
  e.y = y;
  e.oN2 = 1;
  e.oN1 = (int64_t)O * Ho * Wo;
  e.oC = (int64_t)Ho * Wo;
  e.oH = Wo;
  e.O = O;
  e.Ho = ga.Ho;
  e.Wo = ga.Wo;
  e.stride = stride;
  e.crop = crop;
  e.out_len = out_len;
  e.axis_h = axis_h ? 1 : 0;
  gemm_gather(ga, (int64_t)N * ga.Ho * ga.Wo, ph, (int64_t)O * stride, ldo, e);
  DCB_CUDA(cudaFreeAsync(ph, stream()));
}

void dkx_linear(const float *x, int64_t R, int in, const dc_half *weight, int64_t kp, int out,
                const float *bias, float *y) {
  // fp32 rows are the 1x1 "image" [R][in] read as R positions of in channels
  Gather ga{};
  ga.x = x;
  ga.N2 = 1;
  ga.sN1 = (int64_t)in;
  ga.sC = 1;
  ga.sH = 0;
  ga.C = in;
  ga.H = ga.W = 1;
  ga.KH = ga.KW = ga.SH = ga.SW = ga.DH = ga.DW = 1;
  ga.Ho = ga.Wo = 1;
  ga.K = in;
  Epi e;
  e.mode = EPI_ROWS_F32;
  e.bias = bias;
  e.out = y;
  e.ldo = out;
  gemm_gather(ga, R, weight, out, kp, e);
}

}  // extern "C"
