// tcgen05 GEMM family for sm_100a.
//
// One CTA computes a 128 x BN output tile with a warp-specialised pipeline:
//   warps 0-3  A-operand producers when A is gathered (implicit im2col from fp32
//              activations, converted to fp16 with round-to-nearest-even as the reference's
//              dk_im2col_half does), then the epilogue (TMEM -> registers -> fused
//              bias / GELU / GLU / residual / layout transform -> global);
//   warp 4     TMA producer (B tiles, and A tiles when A is already fp16 rows);
//   warp 5     TMEM allocator; lane 0 issues tcgen05.mma (M=128, N=BN, K=16 steps) and
//              tcgen05.commit, which frees operand stages and finally signals the epilogue.
// Operands use the K-major SWIZZLE_128B layout (see umma.cuh); a STAGES-deep smem ring
// (mbarrier full/empty pairs) overlaps loads with MMAs.
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
  int tmem_cols;
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
      int o = (int)(n / e.stride), r = (int)(n - (int64_t)o * e.stride);
      if (o >= e.O) return;
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
                                                 float va, float vb) {
  if (o >= e.O) return;
  float a = va + (e.bias ? e.bias[o] : 0.f);
  float b = vb + (e.bias ? e.bias[e.O + o] : 0.f);
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
constexpr int kProdWarps = 8;             // warps 0-7: gather producers, then epilogue
constexpr int kTmaWarp = kProdWarps;      // warp 8
constexpr int kMmaWarp = kProdWarps + 1;  // warp 9
constexpr int kThreads = 32 * (kProdWarps + 2);

template <int BN, bool GATHER>
__global__ void __launch_bounds__(kThreads, 2)
    k_umma(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const Shape s, const Gather g, const Epi e) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr uint32_t kBTileBytes = BN * 128;
  const int stages = s.stages;
  uint8_t *sA = smem;
  uint8_t *sB = smem + stages * kATileBytes;
  uint64_t *full = (uint64_t *)(sB + stages * kBTileBytes);
  uint64_t *empty = full + stages;
  uint64_t *done = empty + stages;
  uint32_t *tslot = (uint32_t *)(done + 1);
  int2 *ktab = (int2 *)(tslot + 2);

  // a fault recorded by an earlier kernel: end this grid at once (uniform CTA decision)
  __shared__ uint32_t s_abort;
  if (threadIdx.x == 0) s_abort = fault_pending() ? 1u : 0u;
  __syncthreads();
  if (s_abort) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.y, bz = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.x * kBM;
  const int n0 = nt * BN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; i++) {
      mbar_init(&full[i], 1 + (GATHER ? kProdWarps : 0));
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tslot, (uint32_t)s.tmem_cols);
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
      const uint32_t bytes = kBTileBytes + (GATHER ? 0u : kATileBytes);
      const int cA = s.a_shared ? 0 : bz, cB = s.b_shared ? 0 : bz;
      for (int kb = 0; kb < s.nkb; kb++) {
        const int st = kb % stages;
        const uint32_t ph = (uint32_t)(kb / stages) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, kFaultEmpty)) break;
        mbar_expect_tx(&full[st], bytes);
        tma_load_3d(sB + st * kBTileBytes, &tmB, &full[st], kb * kBK, n0, cB);
        if (!GATHER) tma_load_3d(sA + st * kATileBytes, &tmA, &full[st], kb * kBK, (int)m0, cA);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(kBM, BN);
      for (int kb = 0; kb < s.nkb; kb++) {
        const int st = kb % stages;
        const uint32_t ph = (uint32_t)(kb / stages) & 1u;
        if (!mbar_wait(&full[st], ph, kFaultFull)) break;
        tc_fence_after();
        const uint64_t ad = sw128_desc(smem_u32(sA + st * kATileBytes));
        const uint64_t bd = sw128_desc(smem_u32(sB + st * kBTileBytes));
#pragma unroll
        for (int k = 0; k < kBK / 16; k++) {
          // +32 bytes per K=16 step inside the 128-byte swizzle row (>> 4 = 2)
          umma_f16(tmem, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[st]);
      }
      umma_commit(done);
    }
  } else {
    // ---- warps 0-7: warp w serves TMEM lane quarter (w & 3) = tile rows 32(w&3)..+31
    // and half (w >> 2) of the K columns (gather) / accumulator columns (epilogue)
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;  // tile row 0..127
    if (GATHER) {
      const int64_t p = m0 + r;
      int64_t base = 0;
      int h0 = -(1 << 20), w0 = 0;
      if (p < s.M) {
        const int64_t hw = (int64_t)g.Ho * g.Wo;
        const int64_t n = p / hw, rem = p - n * hw;
        const int ho = (int)(rem / g.Wo), wo = (int)(rem - (int64_t)ho * g.Wo);
        const int64_t n1 = n / g.N2, n2 = n - n1 * g.N2;
        h0 = ho * g.SH - g.PH;
        w0 = wo * g.SW - g.PW;
        base = n1 * g.sN1 + n2 * g.sN2 + (int64_t)h0 * g.sH + w0;
      }
      const float *__restrict__ x = g.x;
      const float *__restrict__ x2 = g.x2;
      constexpr int KH2 = kBK / 2;  // 32 columns of each K block per thread
      for (int kb = 0; kb < s.nkb; kb++) {
        const int st = kb % stages;
        const uint32_t ph = (uint32_t)(kb / stages) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, kFaultEmpty)) break;
        const int2 *kt = ktab + kb * kBK + half * KH2;
        float v[KH2];
        if (x2) {
#pragma unroll
          for (int i = 0; i < KH2; i++) {
            const int2 t = kt[i];
            const int hh = h0 + (t.y & 0xffff), ww = w0 + (t.y >> 16);
            const bool ok = (unsigned)hh < (unsigned)g.H && (unsigned)ww < (unsigned)g.W;
            v[i] = ok ? __ldg(x + base + t.x) + __ldg(x2 + base + t.x) : 0.f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < KH2; i++) {
            const int2 t = kt[i];
            const int hh = h0 + (t.y & 0xffff), ww = w0 + (t.y >> 16);
            const bool ok = (unsigned)hh < (unsigned)g.H && (unsigned)ww < (unsigned)g.W;
            v[i] = ok ? __ldg(x + base + t.x) : 0.f;
          }
        }
        const uint32_t a_base = smem_u32(sA + st * kATileBytes);
#pragma unroll
        for (int c = 0; c < 4; c++) {
          st_shared_v4(a_base + sw128_off(r, half * 4 + c), pack_h2(v[8 * c], v[8 * c + 1]),
                       pack_h2(v[8 * c + 2], v[8 * c + 3]), pack_h2(v[8 * c + 4], v[8 * c + 5]),
                       pack_h2(v[8 * c + 6], v[8 * c + 7]));
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[st]);
      }
    }

    mbar_wait(done, 0, kFaultDone);
    tc_fence_after();
    const int64_t m = m0 + r;
    const bool mv = m < s.M;
    const RowInfo ri = mv ? decode_row(e, m) : RowInfo{0, 0, 0, 0, 0};
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    if (e.mode == EPI_CONV) {
      // Staged conv epilogue: chunks of up to 32 output channels go TMEM -> registers
      // (bias, GELU / GLU) -> shared memory [channel][tile row] (the operand buffers are
      // idle once `done` fired), then each warp stores 128 consecutive positions of one
      // channel per step with 16-byte stores (scalar where positions are not contiguous).
      float *stage = (float *)sA + half * (32 * kBM);
      int64_t poff[4];
      bool pv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int64_t mm = m0 + 4 * lane + i;
        pv[i] = mm < s.M;
        poff[i] = 0;
        if (pv[i]) {
          const RowInfo rq = decode_row(e, mm);
          poff[i] = rq.base + (int64_t)rq.ho * e.oH + rq.wo;
        }
      }
      const bool contig = pv[3] && poff[1] == poff[0] + 1 && poff[2] == poff[0] + 2 &&
                          poff[3] == poff[0] + 3;
      const bool glu = e.act == 2;
      const int ncols = glu ? e.glu_half : BN;
      const int per = ncols >= 32 ? ncols / 2 : (half == 0 ? ncols : 0);
      const int c_beg = ncols >= 32 ? half * per : 0;
      const int obase = glu ? nt * e.glu_half : n0;
      for (int c0 = c_beg; c0 < c_beg + per; c0 += 32) {
        const int cw = c_beg + per - c0 >= 32 ? 32 : 16;
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
                const float a = va[i] + (e.bias ? e.bias[o] : 0.f);
                const float b = vb[i] + (e.bias ? e.bias[e.O + o] : 0.f);
                val = a * sigmoid_f(b);
              }
              stage[(sub + i) * kBM + r] = val;
            }
          } else {
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; i++) {
              const int o = obase + c0 + sub + i;
              float val = va[i] + ((e.bias && o < e.O) ? e.bias[o] : 0.f);
              if (e.act == 1) val = gelu_f(val);
              stage[(sub + i) * kBM + r] = val;
            }
          }
        }
        asm volatile("bar.sync %0, %1;" ::"r"(1 + half), "r"(128) : "memory");
        for (int cc = quarter; cc < cw; cc += 4) {
          const int o = obase + c0 + cc;
          if (o < e.O) {
            const float4 v4 = *(const float4 *)(stage + cc * kBM + 4 * lane);
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
        }
        asm volatile("bar.sync %0, %1;" ::"r"(1 + half), "r"(128) : "memory");
      }
    } else {
      constexpr int PER = BN / 2;  // >= 16
      for (int c0 = half * PER; c0 < half * PER + PER; c0 += 16) {
        float v[16];
        tmem_ld16(trow + c0, v);
        tmem_wait_ld();
        if (mv) store_chunk16(e, s, bz, m, (int64_t)n0 + c0, ri, v);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)s.tmem_cols);
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
    const bool glu = e.mode == EPI_CONV && e.act == 2;
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
      store_glu(e, n, ri, acc0, acc1);
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

static int pick_bn(int64_t M, int64_t N, int64_t batch) {
  int bn = 32;
  while (bn < 256 && bn < N) bn *= 2;
  const int64_t mt = (M + kBM - 1) / kBM;
  while (bn > 32 && mt * ((N + bn - 1) / bn) * batch < 148) bn /= 2;
  return bn;
}

int gather_bn(int64_t M, int64_t N, bool glu) {
  int bn = pick_bn(M, N, 1);
  if (glu && bn < 32) bn = 32;
  return bn;
}

template <int BN, bool GATHER>
static void launch_umma(const CUtensorMap &ta, const CUtensorMap &tb, Shape s, const Gather &g,
                        const Epi &e, int64_t mtiles, int ntiles, int64_t batch) {
  const size_t table = GATHER ? (size_t)s.nkb * kBK * sizeof(int2) : 0;
  const size_t stage_bytes = kATileBytes + (size_t)BN * 128;
  // two CTAs per SM (TMEM <= 256 columns and <= ~110 KB shared memory each) so one
  // CTA's gather / epilogue overlaps the other's MMAs
  const size_t budget = 110 * 1024;
  int stages = budget > table + 2048 ? (int)((budget - table - 2048) / stage_bytes) : 0;
  if (stages > 8) stages = 8;
  if (stages > s.nkb + 1) stages = s.nkb + 1;
  if (stages < 2) stages = 2;
  s.stages = stages;
  const size_t smem = 1024 + stages * stage_bytes + (2 * stages + 1) * 8 + 16 + table;
  DCB_REQUIRE(smem <= 226 * 1024, "gemm: shared memory %zu exceeds the per-CTA limit", smem);
  static size_t attr = 0;  // dynamic shared memory opted in so far for this instantiation
  if (smem > attr) {
    DCB_CUDA(cudaFuncSetAttribute(k_umma<BN, GATHER>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = smem;
  }
  s.tmem_cols = BN < 32 ? 32 : BN;
  for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
    DCB_REQUIRE(b0 == 0, "gemm: batch > 65535 on the tensor-core path");
    dim3 grid((unsigned)mtiles, (unsigned)ntiles, (unsigned)(batch < 65535 ? batch : 65535));
    k_umma<BN, GATHER><<<grid, kThreads, smem, stream()>>>(ta, tb, s, g, e);
    DCB_LAUNCHED();
  }
}

template <bool GATHER>
static void dispatch_umma(int bn, const CUtensorMap &ta, const CUtensorMap &tb, Shape s,
                          const Gather &g, const Epi &e, int64_t batch) {
  const int64_t mt = (s.M + kBM - 1) / kBM;
  const int ntl = (int)((s.N + bn - 1) / bn);
  switch (bn) {
    case 32: launch_umma<32, GATHER>(ta, tb, s, g, e, mt, ntl, batch); break;
    case 64: launch_umma<64, GATHER>(ta, tb, s, g, e, mt, ntl, batch); break;
    case 128: launch_umma<128, GATHER>(ta, tb, s, g, e, mt, ntl, batch); break;
    default: launch_umma<256, GATHER>(ta, tb, s, g, e, mt, ntl, batch); break;
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
    // algorithmic work of this call (unpadded extents)
    const double mnk = 2.0 * (double)M * (double)N * (double)K * (double)batch;
    double out_b = (double)M * N * batch * (e.mode == EPI_ROWS_F32 || e.mode == EPI_GEMM ? 4 : 2);
    if (e.res || e.beta != 0.f) out_b *= 2;
    const double in_b = 2.0 * ((double)M * K * (a.stride ? batch : 1) +
                               (double)N * K * (b.stride ? batch : 1));
    TraceScope ts(e.mode == EPI_GEMM ? TR_GEMM : TR_LINEAR, mnk, in_b + out_b, M, N, K);
    gemm_rows_launch(M, N, K, a, b, batch, e, s, g);
  }
}

void gemm_rows_launch(int64_t M, int64_t N, int64_t K, RowsA a, RowsA b, int64_t batch,
                      const Epi &e, Shape s, Gather g) {
  if (!g_opt_simt && K > 0 && batch <= 65535) {
    const int bn = pick_bn(M, N, batch);
    CUtensorMap ta, tb;
    const bool ok =
        encode_map(&ta, a.p, (uint64_t)K, (uint64_t)M, s.a_shared ? 1 : (uint64_t)batch,
                   (uint64_t)a.ld, (uint64_t)a.stride, kBM) &&
        encode_map(&tb, b.p, (uint64_t)K, (uint64_t)N, s.b_shared ? 1 : (uint64_t)batch,
                   (uint64_t)b.ld, (uint64_t)b.stride, (uint32_t)bn);
    if (ok) {
      Epi ev = e;
      ev.vec = vec_ok(e, N) ? 1 : 0;
      dispatch_umma<false>(bn, ta, tb, s, g, ev, batch);
      return;
    }
  }
  launch_simt<false>(a, b, s, g, e, N, batch);
}

void gemm_gather(const Gather &g, int64_t M, const uint16_t *w, int64_t N, int64_t ldw,
                 const Epi &e, int bn_hint) {
  if (M <= 0 || N <= 0) return;
  DCB_REQUIRE(M < (1ll << 31), "conv: too many output positions");
  Shape s{};
  s.M = (int)M;
  s.N = (int)N;
  s.K = g.K;
  s.nkb = (g.K + kBK - 1) / kBK;
  s.a_shared = 1;
  s.b_shared = 1;
  const bool glu = e.mode == EPI_CONV && e.act == 2;
  const int bn = bn_hint ? bn_hint : gather_bn(M, N, glu);
  const double images = (double)M / ((double)g.Ho * g.Wo);
  const double n_alg = e.mode == EPI_CONVTR ? (double)e.O * e.stride : (glu ? 2.0 * e.O : e.O);
  const double out_elems = e.mode == EPI_CONVTR ? (double)M * e.O * e.stride : (double)M * e.O;
  const double x_b = images * g.C * g.H * g.W * 4.0 * (g.x2 ? 2 : 1);
  TraceScope ts(e.mode == EPI_CONVTR ? TR_CONVTR : TR_CONV, 2.0 * M * n_alg * g.K,
                x_b + n_alg * g.K * 2.0 + out_elems * 4.0 * (e.res ? 2 : 1), M, (int64_t)n_alg,
                g.K);
  if (!g_opt_simt) {
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
// -> B[(o, r)][(j', c)] = W[o][r + S (1 - j')][c], j' = 0 reads input q-1, j' = 1 input q.
__global__ void k_convtr_phase(const uint16_t *__restrict__ w, uint16_t *__restrict__ out,
                               int O, int C, int Ktaps, int S, int64_t kp, int64_t ldo) {
  int64_t total = (int64_t)O * S * ldo;
  DCB_GRID_STRIDE(i, total) {
    int64_t row = i / ldo, col = i - row * ldo;
    int o = (int)(row / S), r = (int)(row % S);
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
