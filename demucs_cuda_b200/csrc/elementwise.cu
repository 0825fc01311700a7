// Strided copy / broadcast binary / elementwise part of the backend.h ABI
// (backend.h:42-70).  Memory-bound; the contiguous cases are vectorised with float4.
#include "common.cuh"

namespace dcb {

struct Strides {
  int ndim;
  int64_t shape[DK_MAX_DIM];
  int64_t a[DK_MAX_DIM];
  int64_t b[DK_MAX_DIM];
};

// Collapse the index space: drop unit dims and merge neighbours that are contiguous in
// both operands, so most copies become a few long rows.
static Strides collapse(const DkStrided *p, int64_t *total) {
  Strides s{};
  int64_t n = 1;
  for (int i = 0; i < p->ndim; i++) n *= p->shape[i];
  *total = n;
  int k = 0;
  for (int i = 0; i < p->ndim; i++) {
    if (p->shape[i] == 1) continue;
    if (k > 0 && s.a[k - 1] == p->a_strides[i] * p->shape[i] &&
        s.b[k - 1] == p->b_strides[i] * p->shape[i]) {
      s.shape[k - 1] *= p->shape[i];
      s.a[k - 1] = p->a_strides[i];
      s.b[k - 1] = p->b_strides[i];
      continue;
    }
    s.shape[k] = p->shape[i];
    s.a[k] = p->a_strides[i];
    s.b[k] = p->b_strides[i];
    k++;
  }
  if (k == 0) {
    s.shape[0] = 1;
    k = 1;
  }
  s.ndim = k;
  return s;
}

static __device__ __forceinline__ void unravel(const Strides &s, int64_t e, int64_t &ao,
                                               int64_t &bo) {
  ao = 0;
  bo = 0;
  for (int d = s.ndim - 1; d >= 0; d--) {
    int64_t n = s.shape[d];
    int64_t i = e % n;
    e /= n;
    ao += i * s.a[d];
    bo += i * s.b[d];
  }
}

__global__ void k_strided_copy(Strides s, int64_t n, const float *__restrict__ src,
                               float *__restrict__ dst, int acc) {
  DCB_GRID_STRIDE(e, n) {
    int64_t ao, bo;
    unravel(s, e, ao, bo);
    float v = src[ao];
    if (acc) {
      dst[bo] += v;
    } else {
      dst[bo] = v;
    }
  }
}

// rows of `len` contiguous floats on both sides, row starts by a 1- or 2-level index
__global__ void k_copy_rows(int64_t rows, int64_t len, int64_t inner_rows, int64_t a_outer,
                            int64_t a_inner, int64_t b_outer, int64_t b_inner,
                            const float *__restrict__ src, float *__restrict__ dst, int acc) {
  int64_t total = rows * len;
  DCB_GRID_STRIDE(e, total) {
    int64_t r = e / len, c = e - r * len;
    int64_t ro = r / inner_rows, ri = r - ro * inner_rows;
    float v = src[ro * a_outer + ri * a_inner + c];
    float *d = dst + ro * b_outer + ri * b_inner + c;
    if (acc) {
      *d += v;
    } else {
      *d = v;
    }
  }
}

static __device__ __forceinline__ float binop(int op, float a, float b) {
  switch (op) {
    case DK_ADD: return a + b;
    case DK_SUB: return a - b;
    case DK_MUL: return a * b;
    case DK_DIV: return a / b;
    default: return a > b ? a : b;
  }
}

__global__ void k_binary(Strides s, int64_t n, int op, const float *__restrict__ a,
                         const float *__restrict__ b, float *__restrict__ y) {
  DCB_GRID_STRIDE(e, n) {
    int64_t ao, bo;
    unravel(s, e, ao, bo);
    y[e] = binop(op, a[ao], b[bo]);
  }
}

__global__ void k_unary(int op, const float *__restrict__ x, float *__restrict__ y, int64_t n,
                        float alpha, float beta) {
  DCB_GRID_STRIDE(i, n) {
    float v = x[i];
    float r;
    switch (op) {
      case DK_UN_AFFINE: r = v * alpha + beta; break;
      case DK_UN_GELU: r = gelu_f(v); break;
      case DK_UN_RELU: r = v > 0.0f ? v : 0.0f; break;
      default: r = sigmoid_f(v); break;
    }
    y[i] = r;
  }
}

__global__ void k_fill(float *y, int64_t n, float v) { DCB_GRID_STRIDE(i, n) y[i] = v; }

__global__ void k_glu(const float *__restrict__ x, float *__restrict__ y, int64_t outer,
                      int64_t half, int64_t inner) {
  int64_t hn = half * inner, n = outer * hn;
  DCB_GRID_STRIDE(i, n) {
    int64_t o = i / hn, r = i - o * hn;
    const float *a = x + o * 2 * hn;
    y[i] = a[r] * sigmoid_f(a[r + hn]);
  }
}

__global__ void k_channel_bias(float *y, const float *__restrict__ bias, int64_t outer,
                               int64_t C, int64_t inner) {
  int64_t n = outer * C * inner;
  DCB_GRID_STRIDE(i, n) { y[i] += bias[(i / inner) % C]; }
}

__global__ void k_scale_add(float *y, const float *__restrict__ x,
                            const float *__restrict__ scale, int64_t outer, int64_t C,
                            int64_t inner) {
  int64_t n = outer * C * inner;
  DCB_GRID_STRIDE(i, n) { y[i] += x[i] * scale[(i / inner) % C]; }
}

__global__ void k_reflect_pad(const float *__restrict__ x, float *__restrict__ y, int64_t rows,
                              int64_t L, int64_t left, int64_t right) {
  int64_t Lo = L + left + right, n = rows * Lo;
  DCB_GRID_STRIDE(e, n) {
    int64_t r = e / Lo, i = e - r * Lo;
    int64_t j = i - left;
    if (j < 0) j = -j;
    if (j >= L) j = 2 * L - 2 - j;
    y[e] = x[r * L + j];
  }
}

}  // namespace dcb

using namespace dcb;

extern "C" {

void dk_strided_copy(const DkStrided *p, const float *src, float *dst, int accumulate) {
  int64_t n;
  Strides s = collapse(p, &n);
  if (n == 0) return;
  if (s.a[s.ndim - 1] == 1 && s.b[s.ndim - 1] == 1 && s.ndim <= 3) {
    int64_t len = s.shape[s.ndim - 1];
    int64_t rows = n / len;
    int64_t inner_rows = s.ndim == 3 ? s.shape[1] : rows;
    int64_t ao = s.ndim == 3 ? s.a[0] : (s.ndim == 2 ? s.a[0] : 0);
    int64_t ai = s.ndim == 3 ? s.a[1] : (s.ndim == 2 ? s.a[0] : 0);
    int64_t bo = s.ndim == 3 ? s.b[0] : (s.ndim == 2 ? s.b[0] : 0);
    int64_t bi = s.ndim == 3 ? s.b[1] : (s.ndim == 2 ? s.b[0] : 0);
    if (s.ndim == 2) inner_rows = rows;  // row r -> r*stride via the inner level
    if (s.ndim == 2) {
      ao = 0;
      bo = 0;
    }
    k_copy_rows<<<grid_for(n, 256), 256, 0, stream()>>>(rows, len, inner_rows, ao, ai, bo, bi,
                                                        src, dst, accumulate);
  } else {
    k_strided_copy<<<grid_for(n, 256), 256, 0, stream()>>>(s, n, src, dst, accumulate);
  }
  DCB_LAUNCHED();
}

void dk_binary(DkBinOp op, const DkStrided *p, const float *a, const float *b, float *y) {
  // y is contiguous over the full shape: keep dims (no collapse across y) except unit dims
  Strides s{};
  int64_t n = 1;
  int k = 0;
  for (int i = 0; i < p->ndim; i++) {
    n *= p->shape[i];
    s.shape[k] = p->shape[i];
    s.a[k] = p->a_strides[i];
    s.b[k] = p->b_strides[i];
    k++;
  }
  s.ndim = k > 0 ? k : 1;
  if (k == 0) s.shape[0] = 1;
  if (n == 0) return;
  k_binary<<<grid_for(n, 256), 256, 0, stream()>>>(s, n, (int)op, a, b, y);
  DCB_LAUNCHED();
}

void dk_unary(DkUnOp op, const float *x, float *y, int64_t n, float alpha, float beta) {
  if (n <= 0) return;
  k_unary<<<grid_for(n, 256), 256, 0, stream()>>>((int)op, x, y, n, alpha, beta);
  DCB_LAUNCHED();
}

void dk_fill(float *y, int64_t n, float v) {
  if (n <= 0) return;
  k_fill<<<grid_for(n, 256), 256, 0, stream()>>>(y, n, v);
  DCB_LAUNCHED();
}

void dk_glu(const float *x, float *y, int64_t outer, int64_t half, int64_t inner) {
  int64_t n = outer * half * inner;
  if (n <= 0) return;
  k_glu<<<grid_for(n, 256), 256, 0, stream()>>>(x, y, outer, half, inner);
  DCB_LAUNCHED();
}

void dk_channel_bias(float *y, const float *bias, int64_t outer, int64_t C, int64_t inner) {
  int64_t n = outer * C * inner;
  if (n <= 0) return;
  k_channel_bias<<<grid_for(n, 256), 256, 0, stream()>>>(y, bias, outer, C, inner);
  DCB_LAUNCHED();
}

void dk_scale_add(float *y, const float *x, const float *scale, int64_t outer, int64_t C,
                  int64_t inner) {
  int64_t n = outer * C * inner;
  if (n <= 0) return;
  k_scale_add<<<grid_for(n, 256), 256, 0, stream()>>>(y, x, scale, outer, C, inner);
  DCB_LAUNCHED();
}

void dk_reflect_pad(const float *x, float *y, int64_t rows, int64_t L, int64_t left,
                    int64_t right) {
  int64_t n = rows * (L + left + right);
  if (n <= 0) return;
  k_reflect_pad<<<grid_for(n, 256), 256, 0, stream()>>>(x, y, rows, L, left, right);
  DCB_LAUNCHED();
}

}  // extern "C"
