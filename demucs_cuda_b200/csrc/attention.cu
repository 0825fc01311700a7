// Fused multi-head attention for sm_100a: softmax(Q K^T / sqrt(hd)) V per (batch, head)
// without the score matrix in memory.  Replaces dc_attention's split-heads +
// [GEMM S = Q K^T -> dk_softmax_to_half -> GEMM O = P V] loop (ops.c:390-443,
// attn.cu:26-89).
//
// CTA = 128 query rows of one head, 352 threads, key blocks of 64:
//   warps 0-7  softmax: warp w serves TMEM lane quarter w & 3 (query rows 32 (w & 3) ..
//              +31, one per lane) and column half w >> 2 (32 of the block's 64 keys), so
//              eight warps share the exponentials; the two warps of a quarter exchange
//              their half-block maxima through shared memory and an mbarrier.  Online
//              softmax in fp32 (exp2 domain, running max; the O accumulator stays in TMEM
//              and is rescaled there only when the maximum grows by more than
//              2^kLazyLog2), P written as fp16 into shared memory in the UMMA A-operand
//              layout;
//   warp 8     TMA producer: Q once, then K blocks into a 4-stage ring (a stage is free
//              once S of its block has completed);
//   warp 10    TMA producer: V^T blocks into a 3-stage ring (free once P V of its block
//              has completed);
//   warp 9     TMEM owner; lane 0 issues S = Q K^T (M=128, N=64, K=hd) into one of two
//              TMEM score buffers and O += P V (M=128, N=hd, K=64) from one of two P
//              buffers.  S(j+2) is issued as soon as the softmax warps have read S(j) out
//              of TMEM (s_empty), so it runs while they exponentiate block j.
// TMEM: S0 | S1 | O | row sums (64 + 64 + 64 + 16 columns, 256 allocated); 107 KB of
// shared memory: two CTAs share an SM.  Head dims up to 64 are zero-extended to a multiple of 16 (the MMA K of
// S and N of P V) by TMA out-of-bounds fill; keys past Tk read as zero and are masked out
// of the softmax.
//
// Inputs are fp16 exactly as the reference rounds them (split_heads of the fp32
// projections): Q [BH][Tq][hd], K [BH][Tk][hd], V^T [BH][hd][Tkp].  The reference rounds
// the normalised probabilities to fp16; here the unnormalised exp(s - m_running) is
// rounded (same fp16 operand width) and O is divided at the end by the row sum of those
// fp16 values (accumulated in fp32 by the tensor core).
#include <cudaTypedefs.h>
#include <math.h>

#include "umma.cuh"

namespace dcb {

constexpr int kAttnThreads = 352;
constexpr int kSoftWarps = 8, kKWarp = 8, kMmaWarpA = 9, kVWarp = 10;
constexpr int kQ = 128, kKV = 64, kHD = 64;
constexpr uint32_t kQBytes = kQ * kHD * 2;      // 16 KB
constexpr uint32_t kKBytes = kKV * kHD * 2;     // 8 KB
constexpr uint32_t kVBytes = kHD * kKV * 2;     // 8 KB
constexpr uint32_t kPBytes = kQ * kKV * 2;      // 16 KB per buffer
constexpr int kKStages = 4, kVStages = 3;  // K is released after S, V only after P V
constexpr uint32_t kOnesBytes = 16 * kKV * 2;  // 16 x 64 fp16 ones: the row-sum operand
constexpr uint32_t kRedBytes = 2 * 2 * kQ * 4;  // half-block maxima [block parity][half][row]
// + 512: the 32 mbarriers (256 B), the TMEM slot and the abort flag
constexpr size_t kAttnSmem = kQBytes + kKStages * kKBytes + kVStages * kVBytes + 2 * kPBytes +
                             kOnesBytes + kRedBytes + 512;
constexpr int kSumCol = 64;       // TMEM column (after O) of the row sums of P
constexpr float kLazyLog2 = 2.0f; // rescale when a block maximum exceeds the running one by 4x

struct AttnArgs {
  int Tq, Tk, H, hd, BH;
  float scale;
  uint16_t *o16;  // [B][Tq][H*hd] fp16 (may be null)
  float *o32;     // [B][Tq][H*hd] fp32 (may be null)
};


// 2^x of two fp16 values (PTX ex2.approx.f16x2)
static __device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// (x0, x1) = (a0, a1) * s + c by one packed fp32 FMA (sm_100 fma.rn.f32x2; each lane rounds
// as fmaf does)
static __device__ __forceinline__ void fma2(float &x0, float &x1, float a0, float a1, float s,
                                            float c) {
  asm("{\n\t.reg .b64 ra, rs, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rs, {%4, %4};\n\t"
      "mov.b64 rc, {%5, %5};\n\t"
      "fma.rn.f32x2 rd, ra, rs, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(x0), "=f"(x1)
      : "f"(a0), "f"(a1), "f"(s), "f"(c));
}
// max of three floats in one instruction (sm_100 three-input max.f32)
static __device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}


__global__ void __launch_bounds__(kAttnThreads, 2)
    k_flash_attn(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  // dynamic shared memory only (no static), 1024-aligned for the SW128 operand tiles, so
  // two CTAs fit on one SM
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *sQ = smem;
  uint8_t *sK = sQ + kQBytes;
  uint8_t *sV = sK + kKStages * kKBytes;
  uint8_t *sP = sV + kVStages * kVBytes;
  uint8_t *sOnes = sP + 2 * kPBytes;
  float *sRed = (float *)(sOnes + kOnesBytes);
  uint64_t *bar = (uint64_t *)((uint8_t *)sRed + kRedBytes);
  uint64_t *q_full = bar;
  uint64_t *k_full = bar + 1;              // [kKStages]
  uint64_t *k_empty = k_full + kKStages;   // [kKStages]
  uint64_t *v_full = k_empty + kKStages;   // [kVStages]
  uint64_t *v_empty = v_full + kVStages;   // [kVStages]
  uint64_t *s_full = v_empty + kVStages;   // [2] score buffers computed
  uint64_t *s_empty = s_full + 2;          // [2] score buffers read by the softmax warps
  uint64_t *p_full = s_empty + 2;          // [2] P buffers written
  uint64_t *p_empty = p_full + 2;          // [2] PV of a P buffer complete
  uint64_t *o_full = p_empty + 2;
  uint64_t *xch = o_full + 1;              // [4 quarters][2] half-block maxima written
  uint32_t *tslot = (uint32_t *)(xch + 8);
  uint32_t *s_abort = tslot + 1;

  // a fault recorded by an earlier kernel, or a misaligned window: end this grid at once
  if (threadIdx.x == 0) {
    uint32_t ab = fault_pending() ? 1u : 0u;
    if (smem_u32(smem) & 1023u) {
      atomicOr(&g_dev_fault, kFaultAttn);
      ab = 1u;
    }
    *s_abort = ab;
  }
  __syncthreads();
  if (*s_abort) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, bh = blockIdx.y;
  const int q0 = qt * kQ;
  const int nkv = (a.Tk + kKV - 1) / kKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKStages; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; i++) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kSoftWarps);
      mbar_init(&p_full[i], kSoftWarps);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(o_full, 1);
    for (int i = 0; i < 8; i++) mbar_init(&xch[i], 2);
    fence_mbar_init();
  }
  if (warp == kMmaWarpA) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  if (threadIdx.x < kOnesBytes / 16) {
    // fp16 1.0 everywhere (the swizzled layout of a constant tile is the tile itself),
    // published to the tensor core's async proxy
    st_shared_v4(smem_u32(sOnes) + threadIdx.x * 16, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u,
                 0x3C003C00u);
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tO = tmem + 2 * kKV;

  if (warp == kKWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      mbar_expect_tx(q_full, kQBytes);
      tma_load_3d(sQ, &tmQ, q_full, 0, q0, bh);
      for (int j = 0; j < nkv; j++) {
        const int st = j % kKStages;
        const uint32_t ph = (uint32_t)(j / kKStages) & 1u;
        if (!mbar_wait_sleep(&k_empty[st], ph ^ 1u, kFaultAttn)) break;
        mbar_expect_tx(&k_full[st], kKBytes);
        tma_load_3d(sK + st * kKBytes, &tmK, &k_full[st], 0, j * kKV, bh);
      }
    }
  } else if (warp == kVWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmV);
      for (int j = 0; j < nkv; j++) {
        const int st = j % kVStages;
        const uint32_t ph = (uint32_t)(j / kVStages) & 1u;
        if (!mbar_wait_sleep(&v_empty[st], ph ^ 1u, kFaultAttn)) break;
        mbar_expect_tx(&v_full[st], kVBytes);
        tma_load_3d(sV + st * kVBytes, &tmV, &v_full[st], j * kKV, 0, bh);
      }
    }
  } else if (warp == kMmaWarpA) {
    if (lane == 0) {
      // the head dim rounded up to the MMA granule: K steps of S, N of P V
      const int hd16 = (a.hd + 15) / 16;
      const uint32_t id_s = idesc_f16_f32(kQ, kKV);
      const uint32_t id_o = idesc_f16_f32(kQ, 16 * hd16);
      const uint32_t id_l = idesc_f16_f32(kQ, 16);
      const uint64_t od = sw128_desc(smem_u32(sOnes));
      bool ok = mbar_wait_sleep(q_full, 0, kFaultAttn);
      const uint64_t qd = sw128_desc(smem_u32(sQ));
      // S(j) = Q K(j)^T into score buffer j & 1; K stage released when it completes
      auto issue_s = [&](int j) -> bool {
        const int st = j % kKStages;
        if (!mbar_wait_sleep(&k_full[st], (uint32_t)(j / kKStages) & 1u, kFaultAttn))
          return false;
        tc_fence_after();
        const uint64_t kd = sw128_desc(smem_u32(sK + st * kKBytes));
        const uint32_t dS = tmem + (uint32_t)(j & 1) * kKV;
        for (int k = 0; k < hd16; k++) umma_f16(dS, qd + 2u * k, kd + 2u * k, id_s, k > 0);
        umma_commit(&s_full[j & 1]);
        umma_commit(&k_empty[st]);
        return true;
      };
      for (int j = 0; j < nkv && j < 2 && ok; j++) ok = issue_s(j);
      for (int j = 0; j < nkv && ok; j++) {
        // S(j + 2) into buffer j & 1 as soon as the softmax warps have read S(j)
        if (j + 2 < nkv) {
          if (!mbar_wait_sleep(&s_empty[j & 1], (uint32_t)(j >> 1) & 1u, kFaultAttn)) break;
          tc_fence_after();
          if (!(ok = issue_s(j + 2))) break;
        }
        // O lives in TMEM across all key blocks
        const int sv = j % kVStages;
        if (!mbar_wait_sleep(&p_full[j & 1], (uint32_t)(j >> 1) & 1u, kFaultAttn)) break;
        if (!mbar_wait_sleep(&v_full[sv], (uint32_t)(j / kVStages) & 1u, kFaultAttn)) break;
        tc_fence_after();
        const uint64_t pd = sw128_desc(smem_u32(sP + (j & 1) * kPBytes));
        const uint64_t vd = sw128_desc(smem_u32(sV + sv * kVBytes));
        // O += P(j) V(j); the row sums of the fp16 P accumulate in column kSumCol
#pragma unroll
        for (int k = 0; k < kKV / 16; k++) {
          const uint32_t acc = (j > 0 || k > 0) ? 1u : 0u;
          umma_f16(tO, pd + 2u * k, vd + 2u * k, id_o, acc);
          umma_f16(tO + kSumCol, pd + 2u * k, od + 2u * k, id_l, acc);
        }
        umma_commit(&p_empty[j & 1]);
        umma_commit(&v_empty[sv]);
      }
      umma_commit(o_full);
    }
  } else {
    // softmax warps: warp w serves query rows 32 q .. 32 q + 31 (q = w & 3, the TMEM lane
    // quarter it may access), one per lane, and columns 32 h .. 32 h + 31 (h = w >> 2) of
    // each 64-key block; exp2 domain (scores scaled by scale * log2 e).  The running maximum
    // m is only raised, and O (in TMEM) rescaled, when a block's maximum exceeds it by more
    // than kLazyLog2: probabilities stay <= 4 and most blocks need no rescale.  The block
    // maximum is the larger of the two warps' half-block maxima (exchanged through shared
    // memory under an mbarrier of the warp pair), so both warps keep the same m.
    // P = 2^(s - m) is evaluated two at a time in fp16 (packed fp32 FMA for the exponent,
    // ex2.approx.f16x2 of its fp16 rounding: at most 2^-11 * 2 error in the exponent of the
    // largest probabilities), the operand precision P V uses anyway; the row sums come from
    // the tensor core (P times a ones tile).  tcgen05.ld / st are warp-collective
    // (.sync.aligned): every decision in front of a TMEM access is warp-uniform (a wait's
    // outcome through warp_all, the rescale through __any_sync).
    const int q = warp & 3, h = warp >> 2;
    const int r = q * 32 + lane;
    const uint32_t lrow = (uint32_t)(q * 32) << 16;
    const float sl2 = a.scale * 1.4426950408889634f;
    float m_run = -INFINITY;
    bool ok = true;
    for (int j = 0; j < nkv && ok; j++) {
      if (!warp_all(mbar_wait_sleep(&s_full[j & 1], (uint32_t)(j >> 1) & 1u, kFaultAttn))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[32];
      const uint32_t tS = tmem + (uint32_t)(j & 1) * kKV + (uint32_t)h * 32 + lrow;
      tmem_ld16(tS, *(float(*)[16])v);
      tmem_ld16(tS + 16, *(float(*)[16])(v + 16));
      tmem_wait_ld();
      // score buffer j & 1 may take S(j + 2) once all eight warps have read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[j & 1]);
      const int kbase = j * kKV + h * 32;
      if (kbase + 32 > a.Tk) {
#pragma unroll
        for (int i = 0; i < 32; i++)
          if (kbase + i >= a.Tk) v[i] = -INFINITY;
      }
      // half-block maximum by three-input max, four independent chains
      float m4[4];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const float *vc = v + 8 * c;
        m4[c] = fmaxf(max3(max3(vc[0], vc[1], vc[2]), vc[3], vc[4]), max3(vc[5], vc[6], vc[7]));
      }
      const float mh = fmaxf(max3(m4[0], m4[1], m4[2]), m4[3]);
      // exchange with the other warp of this quarter through shared memory; the pair's
      // mbarrier (two arrivals, alternating buffers: block j + 2 reuses this one) orders the
      // writes before the reads, and its wait is bounded like every other
      float *rb = sRed + (j & 1) * 2 * kQ;
      rb[h * kQ + r] = mh;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xch[q * 2 + (j & 1)]);
      if (!warp_all(mbar_wait(&xch[q * 2 + (j & 1)], (uint32_t)(j >> 1) & 1u, kFaultAttn))) {
        ok = false;
        break;
      }
      const float ms = fmaxf(mh, rb[(1 - h) * kQ + r]) * sl2;
      // raise this row's maximum when its block maximum exceeds it by more than kLazyLog2;
      // the warp rescales when any of its rows does (rows that keep their maximum scale by 1)
      const bool raise = ms > m_run + kLazyLog2;
      if (__any_sync(0xffffffffu, raise)) {
        if (j > 0) {
          // rescale this warp's half of the accumulated O rows (and, for h = 0, the running
          // sums) to the new maxima once PV(j-1) has completed
          if (!warp_all(mbar_wait(&p_empty[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u,
                                  kFaultAttn))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha = raise ? exp2f(m_run - ms) : 1.0f;
#pragma unroll
          for (int c = 0; c < 48; c += 16) {
            // h = 0: O columns 0..31 and the sums; h = 1: O columns 32..63
            if (c == 32 && h == 1) break;
            const uint32_t col = c < 32 ? (uint32_t)(h * 32 + c) : (uint32_t)kSumCol;
            float ov[16];
            tmem_ld16(tO + lrow + col, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; i++) ov[i] *= alpha;
            tmem_st16(tO + lrow + col, ov);
          }
          tmem_wait_st();
        }
        if (raise) m_run = ms;
      }
      // P buffer j & 1 is free once PV(j-2) has completed
      if (j >= 2 && !warp_all(mbar_wait(&p_empty[j & 1], (uint32_t)((j - 2) >> 1) & 1u,
                                        kFaultAttn))) {
        ok = false;
        break;
      }
      uint32_t w[16];
      const float nm = -m_run;
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        float x0, x1;
        fma2(x0, x1, v[i], v[i + 1], sl2, nm);
        w[i >> 1] = ex2_h2(pack_h2(x0, x1));
      }
      // this half's four 16-byte chunks (8 keys each) of row r, SW128 A-operand layout
      const uint32_t prow = smem_u32(sP + (j & 1) * kPBytes);
#pragma unroll
      for (int c = 0; c < 4; c++)
        st_shared_v4(prow + sw128_off(r, 4 * h + c), w[4 * c], w[4 * c + 1], w[4 * c + 2],
                     w[4 * c + 3]);
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j & 1]);
    }
    // normalise and store this warp's half of the finished O row
    if (warp_all(ok && mbar_wait(o_full, 0, kFaultAttn))) {
      tc_fence_after();
      const int t = q0 + r;
      float lsum[16];
      tmem_ld16(tO + lrow + kSumCol, lsum);
      tmem_wait_ld();
      const float inv = 1.0f / lsum[0];
      const int b = bh / a.H, hh = bh - b * a.H;
      const int64_t D = (int64_t)a.H * a.hd;
      const int64_t off = ((int64_t)b * a.Tq + t) * D + (int64_t)hh * a.hd;
#pragma unroll
      for (int c = h * 32; c < h * 32 + 32; c += 16) {
        float ov[16];
        tmem_ld16(tO + lrow + c, ov);
        tmem_wait_ld();
        if (t < a.Tq) {
#pragma unroll
          for (int i = 0; i < 16; i++) {
            if (c + i < a.hd) {
              const float val = ov[i] * inv;
              if (a.o16) a.o16[off + c + i] = f2h_bits(val);
              if (a.o32) a.o32[off + c + i] = val;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarpA) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ------------------------------------------------------------ CUDA-core reference kernel
// One warp per (query, head); exact reference numerics: max over scaled scores, sum of
// exps in double, P = fp16(exp(v - max) * (1/sum)), O = sum P V in fp32.
__global__ void k_attn_simt(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                            const uint16_t *__restrict__ vt, AttnArgs a, int64_t Tkp) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)a.BH * a.Tq) return;
  const int bh = (int)(gw / a.Tq), t = (int)(gw - (int64_t)bh * a.Tq);
  const uint16_t *qr = q + ((int64_t)bh * a.Tq + t) * a.hd;
  float qv[64];
  for (int d = 0; d < a.hd; d++) qv[d] = h2f_bits(qr[d]);
  auto score = [&](int j) {
    const uint16_t *kr = k + ((int64_t)bh * a.Tk + j) * a.hd;
    float s = 0.f;
    for (int d = 0; d < a.hd; d++) s += qv[d] * h2f_bits(kr[d]);
    return s * a.scale;
  };
  float mx = -INFINITY;
  for (int j = lane; j < a.Tk; j += 32) mx = fmaxf(mx, score(j));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  double sum = 0.0;
  for (int j = lane; j < a.Tk; j += 32) sum += (double)expf(score(j) - mx);
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = (float)(1.0 / sum);
  float acc[64];
  for (int d = 0; d < a.hd; d++) acc[d] = 0.f;
  for (int j = lane; j < a.Tk; j += 32) {
    const float p = h2f_bits(f2h_bits(expf(score(j) - mx) * inv));
    for (int d = 0; d < a.hd; d++) acc[d] += p * h2f_bits(vt[((int64_t)bh * a.hd + d) * Tkp + j]);
  }
  const int b = bh / a.H, h = bh - b * a.H;
  const int64_t D = (int64_t)a.H * a.hd;
  const int64_t off = ((int64_t)b * a.Tq + t) * D + (int64_t)h * a.hd;
  for (int d = 0; d < a.hd; d++) {
    float v = acc[d];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) {
      if (a.o16) a.o16[off + d] = f2h_bits(v);
      if (a.o32) a.o32[off + d] = v;
    }
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 g_enc_attn = nullptr;

static bool map3(CUtensorMap *m, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1) {
  if (!g_enc_attn) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    g_enc_attn = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  }
  if (((uintptr_t)base & 15) || (s1 * 2) % 16 || (s2 * 2) % 16) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1 * 2, s2 * 2};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return g_enc_attn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims,
                    strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// q [BH][Tq][hd], k [BH][Tk][hd], vt [BH][hd][Tkp] fp16 -> o16 / o32 [B][Tq][H*hd]
void flash_attention(const uint16_t *q, const uint16_t *k, const uint16_t *vt, int B, int H,
                     int Tq, int Tk, int hd, int64_t Tkp, uint16_t *o16, float *o32) {
  DCB_REQUIRE(hd <= kHD && hd % 8 == 0, "attention: head dim %d must be a multiple of 8 <= 64",
              hd);
  DCB_REQUIRE(Tkp % 8 == 0 && Tkp >= Tk, "attention: padded key length %lld", (long long)Tkp);
  AttnArgs a;
  a.Tq = Tq;
  a.Tk = Tk;
  a.H = H;
  a.hd = hd;
  a.BH = B * H;
  a.scale = 1.0f / sqrtf((float)hd);
  a.o16 = o16;
  a.o32 = o32;
  TraceScope ts(TR_ATTN, 4.0 * B * H * (double)Tq * Tk * hd,
                2.0 * B * H * hd * (2.0 * Tq + 2.0 * Tk), (int64_t)B * H * Tq, Tk, hd);
  if (!g_opt_simt) {
    CUtensorMap mq, mk, mv;
    bool ok = map3(&mq, q, hd, Tq, (uint64_t)B * H, hd, (uint64_t)Tq * hd, 64, kQ) &&
              map3(&mk, k, hd, Tk, (uint64_t)B * H, hd, (uint64_t)Tk * hd, 64, kKV) &&
              map3(&mv, vt, Tk, hd, (uint64_t)B * H, Tkp, (uint64_t)hd * Tkp, 64, 64);
    if (ok) {
      const size_t smem = kAttnSmem;
      static bool attr = false;
      if (!attr) {
        DCB_CUDA(cudaFuncSetAttribute(k_flash_attn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
        attr = true;
      }
      DCB_REQUIRE(B * H <= 65535, "attention: too many heads");
      dim3 grid((unsigned)((Tq + kQ - 1) / kQ), (unsigned)(B * H));
      k_flash_attn<<<grid, kAttnThreads, smem, stream()>>>(mq, mk, mv, a);
      DCB_LAUNCHED();
      return;
    }
  }
  const int64_t warps = (int64_t)B * H * Tq;
  k_attn_simt<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream()>>>(q, k, vt, a, Tkp);
  DCB_LAUNCHED();
}

// fp32 [B][T][H*hd] -> fp16 [B][H][T][hd] (transpose=0) or [B][H][hd][Tp] (transpose=1)
__global__ void k_heads16(const float *__restrict__ x, uint16_t *__restrict__ y, int B, int T,
                          int H, int hd, int64_t Tp, int transpose) {
  int64_t D = (int64_t)H * hd, n = (int64_t)B * T * D;
  DCB_GRID_STRIDE(i, n) {
    int64_t c = i % D, bt = i / D, t = bt % T, b = bt / T;
    int64_t h = c / hd, d = c % hd;
    uint16_t v = f2h_bits(x[i]);
    if (transpose) {
      y[((b * H + h) * hd + d) * Tp + t] = v;
    } else {
      y[((b * H + h) * T + t) * hd + d] = v;
    }
  }
}

}  // namespace dcb

using namespace dcb;

extern "C" void dkx_attention(const float *q, const float *k, const float *v, int B, int Tq,
                              int Tk, int H, int hd, float *y) {
  if (B <= 0 || Tq <= 0 || Tk <= 0) return;
  const int64_t Tkp = (Tk + 7) / 8 * 8;
  uint16_t *qh = nullptr, *kh = nullptr, *vt = nullptr;
  const size_t nq = (size_t)B * H * Tq * hd, nk = (size_t)B * H * Tk * hd;
  const size_t nv = (size_t)B * H * hd * Tkp;
  DCB_CUDA(cudaMallocAsync(&qh, nq * 2, stream()));
  DCB_CUDA(cudaMallocAsync(&kh, nk * 2, stream()));
  DCB_CUDA(cudaMallocAsync(&vt, nv * 2, stream()));
  DCB_CUDA(cudaMemsetAsync(vt, 0, nv * 2, stream()));
  k_heads16<<<grid_for((int64_t)B * Tq * H * hd, 256), 256, 0, stream()>>>(q, qh, B, Tq, H, hd,
                                                                          0, 0);
  DCB_LAUNCHED();
  k_heads16<<<grid_for((int64_t)B * Tk * H * hd, 256), 256, 0, stream()>>>(k, kh, B, Tk, H, hd,
                                                                          0, 0);
  DCB_LAUNCHED();
  k_heads16<<<grid_for((int64_t)B * Tk * H * hd, 256), 256, 0, stream()>>>(v, vt, B, Tk, H, hd,
                                                                          Tkp, 1);
  DCB_LAUNCHED();
  flash_attention(qh, kh, vt, B, H, Tq, Tk, hd, Tkp, nullptr, y);
  DCB_CUDA(cudaFreeAsync(qh, stream()));
  DCB_CUDA(cudaFreeAsync(kh, stream()));
  DCB_CUDA(cudaFreeAsync(vt, stream()));
}
