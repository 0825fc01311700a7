// Fused multi-head attention for sm_100a: softmax(Q K^T / sqrt(hd)) V per (batch, head)
// without the score matrix in memory.  Replaces dc_attention's split-heads +
// [GEMM S = Q K^T -> dk_softmax_to_half -> GEMM O = P V] loop (ops.c:390-443,
// attn.cu:26-89).
//
// CTA = 128 query rows of one head, 384 threads, key blocks of 64:
//   warps 0-7  softmax: warp w serves TMEM lane quarter q = w & 3 (query rows 32 q .. +31,
//              one per lane) and the key blocks of parity h = w >> 2: the two warps of a
//              quarter take alternate blocks, each with its own running maximum, O
//              accumulator O_h and row sums l_h in TMEM, so a warp has two block times for
//              each of its blocks (all 64 keys of it per thread) and no per-block exchange.
//              Online softmax in fp32 (exp2 domain; O_h is rescaled in TMEM only when the
//              maximum grows by more than 2^kLazyLog2), P written as fp16 into its parity's
//              shared-memory buffer in the UMMA A-operand layout.  At the end the pair
//              exchanges maxima once and combines O = (O_0 a_0 + O_1 a_1) / (l_0 a_0 + l_1 a_1);
//   warp 8     TMA producer: Q once, then K blocks into a 4-stage ring (a stage is free
//              once S of its block has completed); warp 11: V^T blocks into a 3-stage ring
//              (free once P V of its block has completed);
//   warps 9-10 MMA issue (warp 9 also owns the TMEM allocation): lane 0 of warp 9 + h
//              issues, for the blocks j of parity h, S(j) = Q K(j)^T (M=128, N=64, K=hd)
//              into score buffer h and O_h += P(j) V(j), l_h += P(j) 1 (M=128, N=hd / 16,
//              K=64).  S(j + 2) is issued as soon as the parity's warps have read S(j) out
//              of TMEM, so it runs while they exponentiate block j.
// TMEM: S_0 | S_1 | O_0 | O_1 | l_0 | l_1 (64 + 64 + 2 x 16 ceil(hd / 16) + 2 x 16 columns):
// 256 for head dims up to 48 (two CTAs share an SM), 512 above; 109 KB of shared memory.
// Head dims up to 64 are zero-extended to a multiple of 16 (the MMA K of S and N of P V) by
// TMA out-of-bounds fill; keys past Tk read as zero and are masked out of the softmax.
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

constexpr int kAttnThreads = 384;
// one issuing thread per warp (lane 0) for each asynchronous role: warp 8 loads Q and K,
// warp 11 loads V^T, warp 9 (also the TMEM owner) issues parity 0's MMAs and warp 10
// parity 1's, so no two lanes of one warp ever issue a TMA copy, a tcgen05.mma or a
// tcgen05.commit together
constexpr int kSoftWarps = 8, kLoadWarp = 8, kMmaWarpA = 9, kMmaWarpB = 10, kVWarp = 11;
constexpr int kQ = 128, kKV = 64, kHD = 64;
constexpr uint32_t kQBytes = kQ * kHD * 2;      // 16 KB
constexpr uint32_t kKBytes = kKV * kHD * 2;     // 8 KB
constexpr uint32_t kVBytes = kHD * kKV * 2;     // 8 KB
constexpr uint32_t kPBytes = kQ * kKV * 2;      // 16 KB per buffer (one per block parity)
constexpr int kKStages = 4, kVStages = 3;  // K is released after S, V only after P V
constexpr uint32_t kOnesBytes = 16 * kKV * 2;  // 16 x 64 fp16 ones: the row-sum operand
constexpr uint32_t kRedBytes = 2 * kQ * 4;     // final maxima [parity][row]
// + 512: the mbarriers (<= 256 B), the TMEM slot and the abort flag
constexpr size_t kAttnSmem = kQBytes + kKStages * kKBytes + kVStages * kVBytes + 2 * kPBytes +
                             kOnesBytes + kRedBytes + 512;
// one CTA per SM when the accumulators take 512 TMEM columns (head dims above 48)
constexpr size_t kAttnSmemWide = 120 * 1024;
constexpr float kLazyLog2 = 2.0f; // rescale when a block maximum exceeds the running one by 4x

struct AttnArgs {
  int Tq, Tk, H, hd, BH;
  float scale;
  uint16_t *o16;  // [B][Tq][H*hd] fp16 (may be null)
  float *o32;     // [B][Tq][H*hd] fp32 (may be null)
};


// 2^x in fp32 on the special-function unit (PTX ex2.approx.ftz.f32; 2^-inf = +0)
static __device__ __forceinline__ float ex2_f32(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
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
  uint8_t *sP = sV + kVStages * kVBytes;  // [parity] P buffers
  uint8_t *sOnes = sP + 2 * kPBytes;
  float *sRed = (float *)(sOnes + kOnesBytes);
  uint64_t *bar = (uint64_t *)((uint8_t *)sRed + kRedBytes);
  uint64_t *q_full = bar;
  uint64_t *k_full = bar + 1;              // [kKStages]
  uint64_t *k_empty = k_full + kKStages;   // [kKStages]
  uint64_t *v_full = k_empty + kKStages;   // [kVStages]
  uint64_t *v_empty = v_full + kVStages;   // [kVStages]
  uint64_t *s_full = v_empty + kVStages;   // [parity] score buffer computed
  uint64_t *s_empty = s_full + 2;          // [parity] score buffer read by its 4 warps
  uint64_t *p_full = s_empty + 2;          // [parity] P buffer written by its 4 warps
  uint64_t *pv_done = p_full + 2;          // [parity] P V of the parity's latest block done
  uint64_t *o_full = pv_done + 2;          // every MMA done
  uint64_t *xch = o_full + 1;              // [quarter] final maxima written
  uint32_t *tslot = (uint32_t *)(xch + 4);
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
  // TMEM columns: S_0 | S_1 | O_0 | O_1 | l_0 | l_1
  const int hd16 = (a.hd + 15) / 16;
  const uint32_t ow = 16u * (uint32_t)hd16;
  const uint32_t ncols = 2u * kKV + 2u * ow + 32u <= 256u ? 256u : 512u;

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
      mbar_init(&s_empty[i], kSoftWarps / 2);
      mbar_init(&p_full[i], kSoftWarps / 2);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_full, 2);
    for (int i = 0; i < 4; i++) mbar_init(&xch[i], 2);
    fence_mbar_init();
  }
  if (warp == kMmaWarpA) {
    tmem_alloc(tslot, ncols);
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
  const uint32_t tO = tmem + 2 * kKV;     // O_h at tO + h ow
  const uint32_t tL = tO + 2 * ow;        // l_h at tL + 16 h

  if (warp == kLoadWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      mbar_expect_tx(q_full, kQBytes);
      tma_load_3d(sQ, &tmQ, q_full, 0, q0, bh);
      for (int j = 0; j < nkv; j++) {
        const int st = j % kKStages;
        const uint32_t ph = (uint32_t)(j / kKStages) & 1u;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, kFaultAttn)) break;
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
        if (!mbar_wait(&v_empty[st], ph ^ 1u, kFaultAttn)) break;
        mbar_expect_tx(&v_full[st], kVBytes);
        tma_load_3d(sV + st * kVBytes, &tmV, &v_full[st], j * kKV, 0, bh);
      }
    }
  } else if (warp == kMmaWarpA || warp == kMmaWarpB) {
    // two issuing warps, one per block parity h, each on its own chain (S(j + 2) once the
    // parity's warps have read S(j), P V(j) once they have written P(j)), so neither parity
    // waits for the other's softmax
    if (lane == 0) {
      const int h = warp - kMmaWarpA;
      const uint32_t id_s = idesc_f16_f32(kQ, kKV);
      const uint32_t id_o = idesc_f16_f32(kQ, 16 * hd16);
      const uint32_t id_l = idesc_f16_f32(kQ, 16);
      const uint64_t od = sw128_desc(smem_u32(sOnes));
      bool ok = mbar_wait(q_full, 0, kFaultAttn);
      const uint64_t qd = sw128_desc(smem_u32(sQ));
      const uint32_t dS = tmem + (uint32_t)h * kKV;
      // S(j) = Q K(j)^T into score buffer h; K stage released when it completes
      auto issue_s = [&](int j) -> bool {
        const int st = j % kKStages;
        if (!mbar_wait(&k_full[st], (uint32_t)(j / kKStages) & 1u, kFaultAttn)) return false;
        tc_fence_after();
        const uint64_t kd = sw128_desc(smem_u32(sK + st * kKBytes));
        for (int k = 0; k < hd16; k++) umma_f16(dS, qd + 2u * k, kd + 2u * k, id_s, k > 0);
        umma_commit(&s_full[h]);
        umma_commit(&k_empty[st]);
        return true;
      };
      if (ok && h < nkv) ok = issue_s(h);
      uint32_t u = 0;  // this parity's blocks so far
      for (int j = h; j < nkv && ok; j += 2, u++) {
        if (j + 2 < nkv) {
          if (!mbar_wait(&s_empty[h], u & 1u, kFaultAttn)) break;
          tc_fence_after();
          if (!(ok = issue_s(j + 2))) break;
        }
        const int sv = j % kVStages;
        if (!mbar_wait(&p_full[h], u & 1u, kFaultAttn) ||
            !mbar_wait(&v_full[sv], (uint32_t)(j / kVStages) & 1u, kFaultAttn))
          break;
        tc_fence_after();
        const uint64_t pd = sw128_desc(smem_u32(sP + h * kPBytes));
        const uint64_t vd = sw128_desc(smem_u32(sV + sv * kVBytes));
        // O_h += P(j) V(j); the row sums of the fp16 P accumulate in l_h
#pragma unroll
        for (int k = 0; k < kKV / 16; k++) {
          const uint32_t acc = (u > 0 || k > 0) ? 1u : 0u;
          umma_f16(tO + (uint32_t)h * ow, pd + 2u * k, vd + 2u * k, id_o, acc);
          umma_f16(tL + 16u * (uint32_t)h, pd + 2u * k, od + 2u * k, id_l, acc);
        }
        umma_commit(&pv_done[h]);
        umma_commit(&v_empty[sv]);
      }
      umma_commit(o_full);  // (two arrivals: every MMA of both issuing warps)
    }
  } else {
    // softmax warps: warp w serves query rows 32 q .. 32 q + 31 (q = w & 3, the TMEM lane
    // quarter it may access), one per lane, and the key blocks j with j & 1 = h = w >> 2,
    // all 64 keys of each; exp2 domain (scores scaled by scale * log2 e).  The running
    // maximum m is only raised, and O_h (in TMEM) rescaled, when a block's maximum exceeds
    // it by more than kLazyLog2: probabilities stay <= 4 and most blocks need no rescale.
    // P = 2^(s - m) takes its exponent two at a time by packed fp32 FMA, is evaluated in
    // fp32 (ex2.approx) and rounded to fp16, the operand precision P V uses anyway; the row
    // sums come from the tensor core (P times a ones tile).  tcgen05.ld / st are warp-collective
    // (.sync.aligned): every decision in front of a TMEM access is warp-uniform (a wait's
    // outcome through warp_all, the rescale through __any_sync).
    const int q = warp & 3, h = warp >> 2;
    const int r = q * 32 + lane;
    const uint32_t lrow = (uint32_t)(q * 32) << 16;
    const float sl2 = a.scale * 1.4426950408889634f;
    const uint32_t tOh = tO + (uint32_t)h * ow, tLh = tL + 16u * (uint32_t)h;
    const uint32_t prow = smem_u32(sP + h * kPBytes);
    float m_run = -INFINITY;
    bool ok = true;
    uint32_t u = 0;  // this warp's blocks so far
    for (int j = h; j < nkv && ok; j += 2, u++) {
      if (!warp_all(mbar_wait(&s_full[h], u & 1u, kFaultAttn))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[64];
      const uint32_t tS = tmem + (uint32_t)h * kKV + lrow;
#pragma unroll
      for (int c = 0; c < 4; c++) tmem_ld16(tS + 16u * c, *(float(*)[16])(v + 16 * c));
      tmem_wait_ld();
      // score buffer h may take S(j + 2) once the parity's four warps have read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[h]);
      const int kbase = j * kKV;
      if (kbase + kKV > a.Tk) {
#pragma unroll
        for (int i = 0; i < 64; i++)
          if (kbase + i >= a.Tk) v[i] = -INFINITY;
      }
      // block maximum by three-input max, eight independent chains
      float m8[8];
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const float *vc = v + 8 * c;
        m8[c] = fmaxf(max3(max3(vc[0], vc[1], vc[2]), vc[3], vc[4]), max3(vc[5], vc[6], vc[7]));
      }
      const float ms =
          fmaxf(max3(max3(m8[0], m8[1], m8[2]), m8[3], m8[4]), max3(m8[5], m8[6], m8[7])) * sl2;
      // raise this row's maximum when its block maximum exceeds it by more than kLazyLog2;
      // the warp rescales O_h when any of its rows does (rows that keep their maximum scale
      // by 1)
      const bool raise = ms > m_run + kLazyLog2;
      const bool any_raise = __any_sync(0xffffffffu, raise);
      const float alpha = raise && u > 0 ? exp2f(m_run - ms) : 1.0f;
      if (raise) m_run = ms;
      // P = 2^(s sl2 - m) into registers (packed fp16 pairs): the exponentials run while P V
      // of this warp's previous block may still be in flight
      uint32_t w[32];
      const float nm = -m_run;
#pragma unroll
      for (int i = 0; i < 32; i++) {
        float x0, x1;
        fma2(x0, x1, v[2 * i], v[2 * i + 1], sl2, nm);
        w[i] = pack_h2(ex2_f32(x0), ex2_f32(x1));
      }
      // P buffer h and O_h are free once that P V has completed
      if (u > 0 && !warp_all(mbar_wait(&pv_done[h], (u - 1) & 1u, kFaultAttn))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (any_raise && u > 0) {
        // O_h columns, then the row sums l_h (column tLh), 4 columns at a time
#pragma unroll 1
        for (uint32_t c = 0; c < ow + 4u; c += 4u) {
          const uint32_t col = c < ow ? tOh + c : tLh;
          float ov[4];
          tmem_ld4(col + lrow, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 4; i++) ov[i] *= alpha;
          tmem_st4(col + lrow, ov);
        }
        tmem_wait_st();
      }
      // row r's eight 16-byte chunks (8 keys each), SW128 A-operand layout
#pragma unroll
      for (int c = 0; c < 8; c++)
        st_shared_v4(prow + sw128_off(r, c), w[4 * c], w[4 * c + 1], w[4 * c + 2],
                     w[4 * c + 3]);
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[h]);
    }
    // combine the two parities: exchange the row maxima with the quarter's other warp, then
    // O = (O_0 a_0 + O_1 a_1) / (l_0 a_0 + l_1 a_1) with a_h = 2^(m_h - max(m_0, m_1)); a
    // parity with no blocks (nkv = 1) contributes nothing
    sRed[h * kQ + r] = m_run;
    __syncwarp();
    if (lane == 0) mbar_arrive(&xch[q]);
    const bool fin = warp_all(ok && mbar_wait(&xch[q], 0, kFaultAttn) &&
                              mbar_wait(o_full, 0, kFaultAttn));
    if (fin) {
      tc_fence_after();
      const float m_oth = sRed[(1 - h) * kQ + r];
      const bool has0 = nkv >= 1, has1 = nkv >= 2;
      const float m0 = h == 0 ? m_run : m_oth, m1 = h == 0 ? m_oth : m_run;
      const float mm = has1 ? fmaxf(m0, m1) : m0;
      const float a0 = has0 ? exp2f(m0 - mm) : 0.f, a1 = has1 ? exp2f(m1 - mm) : 0.f;
      const float l0 = tmem_ld1(tL + lrow), l1 = tmem_ld1(tL + 16u + lrow);
      tmem_wait_ld();
      const float inv = 1.0f / (l0 * a0 + (has1 ? l1 * a1 : 0.f));
      const int t = q0 + r;
      const int b = bh / a.H, hh = bh - b * a.H;
      const int64_t D = (int64_t)a.H * a.hd;
      const int64_t off = ((int64_t)b * a.Tq + t) * D + (int64_t)hh * a.hd;
      // this warp's half of the columns: h = 0 takes 0..31, h = 1 32..63 (those < hd)
#pragma unroll
      for (int c = h * 32; c < h * 32 + 32; c += 16) {
        if (c >= a.hd) break;
        float o0[16], o1[16];
        tmem_ld16(tO + (uint32_t)c + lrow, o0);
        tmem_ld16(tO + ow + (uint32_t)c + lrow, o1);
        tmem_wait_ld();
        if (t < a.Tq) {
#pragma unroll
          for (int i = 0; i < 16; i++) {
            if (c + i < a.hd) {
              const float val = (o0[i] * a0 + (has1 ? o1[i] * a1 : 0.f)) * inv;
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
    tmem_dealloc(tmem, ncols);
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
      // head dims above 48 take 512 TMEM columns: shared memory then holds one CTA per SM
      const int hd16 = (hd + 15) / 16;
      const size_t smem = 2 * kKV + 32 * hd16 + 32 <= 256 ? kAttnSmem : kAttnSmemWide;
      static bool attr = false;
      if (!attr) {
        DCB_CUDA(cudaFuncSetAttribute(k_flash_attn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)(kAttnSmem > kAttnSmemWide ? kAttnSmem
                                                                      : kAttnSmemWide)));
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
