// RMSNorm / LayerNorm, each with an optional residual add folded in.
//
// HBM-bound: each element of x (and r) is read once and each output written
// once. A row is split over a group of TPR threads that each hold VPT 16-byte
// chunks in registers, so the row is read a single time and the statistics,
// the residual sum and the scaled output all come from registers.
//   n = 128  (per-head q/k norm)  -> 16 threads per row, 16 rows per CTA
//   n = 1280 (ViT LayerNorm)      -> one warp per row, 5 chunks per lane
//   n = 2048 (expert RMSNorm)     -> 128 threads per row, 2 chunks each
//   n = 4096 (LM RMSNorm)         -> 256 threads per row, 2 chunks each
// Few chunks per thread and many threads per row measured fastest (n = 4096 at 24 800
// rows, add+RMSNorm: 136 us with 256 x 2 against 145 us with 128 x 4 and 204 us with
// 64 x 8), and so did four CTAs per SM for the 5-chunk LayerNorm row (125 against 136 us).
// Reductions are warp shuffles, plus a shared-memory step when a row spans
// several warps. Statistics and the scaled output are computed in fp32 and
// rounded to bf16 once, as in the reference kernels (rmsnorm.py:44-51,91-101;
// layernorm.py:43-52,87-100).
//
// The RMSNorm variant with an axpy epilogue (umic_rmsnorm_axpy) writes
// y = base + alpha * normed instead of normed: the flow sampler's Euler update
// x <- x + dt * v, where the velocity v is the expert's final RMSNorm output,
// costs no extra pass over HBM (base read once, y written once, v never stored).
#include "common.cuh"

namespace umic {
namespace {

constexpr int kThreads = 256;

struct NormArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* r;  // residual, add variants only
  const void* w;
  const void* b;  // LayerNorm bias
  __nv_bfloat16* y;  // normed output
  __nv_bfloat16* s;  // summed output, add variants only
  const __nv_bfloat16* base;  // axpy epilogue: y = base + alpha * normed
  int64_t sx, sr, sy, ss, sb;
  float alpha;
  int64_t rows;
  int n;
  int w_dtype;
  float eps;
};

// Sum over the TPR threads of one row group. For TPR > 32 the group spans
// several warps and the partials meet in shared memory.
template <int TPR>
__device__ __forceinline__ float group_sum(float v, float* red) {
  constexpr int kLanes = TPR < 32 ? TPR : 32;
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if constexpr (TPR > 32) {
    constexpr int kWarpsPerRow = TPR / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = threadIdx.x / TPR;
    __syncthreads();  // red may still hold the previous reduction
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kWarpsPerRow; ++i) t += red[grp * kWarpsPerRow + i];
    v = t;
  }
  return v;
}

// Up to 5 chunks per thread the row fits in 64 registers: four CTAs (1024 threads) per SM.
template <int TPR, int VPT, bool kAdd, bool kLayerNorm, bool kAxpy = false>
__global__ void __launch_bounds__(kThreads, VPT <= 5 ? 4 : 1) norm_vec_kernel(NormArgs a) {
  allow_dependent_launch();
  wait_prerequisite();
  constexpr int kRowsPerCta = kThreads / TPR;
  __shared__ float red[kThreads / 32];
  const int sub = threadIdx.x % TPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerCta + threadIdx.x / TPR;
  const bool row_ok = row < a.rows;
  const int nchunk = a.n >> 3;

  float v[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = sub + i * TPR;
    if (row_ok && c < nchunk) {
      unpack8(ld_stream(a.x + row * a.sx + c * 8), v[i]);
      if constexpr (kAdd) {
        float t[8];
        unpack8(ld_stream(a.r + row * a.sr + c * 8), t);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += t[j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    }
  }

  if constexpr (kAdd) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = sub + i * TPR;
      if (row_ok && c < nchunk) st_vec(a.s + row * a.ss + c * 8, pack8(v[i]));
    }
  }

  const float inv_n = 1.f / static_cast<float>(a.n);
  float mean = 0.f;
  if constexpr (kLayerNorm) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) t += v[i][j];
    mean = group_sum<TPR>(t, red) * inv_n;
  }
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const bool valid = (sub + i * TPR) < nchunk;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d = kLayerNorm ? (valid ? v[i][j] - mean : 0.f) : v[i][j];
      q += d * d;
    }
  }
  const float rstd = rsqrtf(group_sum<TPR>(q, red) * inv_n + a.eps);

  if (!row_ok) return;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = sub + i * TPR;
    if (c >= nchunk) continue;
    float w[8], o[8];
    load_w8(a.w, a.w_dtype, c * 8, w);
    if constexpr (kLayerNorm) {
      float bb[8];
      load_w8(a.b, a.w_dtype, c * 8, bb);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (v[i][j] - mean) * rstd * w[j] + bb[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * rstd * w[j];
    }
    if constexpr (kAxpy) {
      float xb[8];
      unpack8(ld_stream(a.base + row * a.sb + c * 8), xb);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = fmaf(a.alpha, o[j], xb[j]);
    }
    st_vec(a.y + row * a.sy + c * 8, pack8(o));
  }
}

// Any n up to kScalarMaxN, any alignment: one CTA per row, the fp32 row
// (after the residual add) staged in shared memory so x / r are read once.
constexpr int kScalarMaxN = 16384;

template <bool kAdd, bool kLayerNorm, bool kAxpy = false>
__global__ void __launch_bounds__(kThreads) norm_scalar_kernel(NormArgs a) {
  allow_dependent_launch();
  extern __shared__ float srow[];
  __shared__ float red[kThreads / 32];
  const int64_t row = blockIdx.x;
  const int n = a.n;
  float t = 0.f;
  for (int j = threadIdx.x; j < n; j += kThreads) {
    float v = bf(a.x[row * a.sx + j]);
    if constexpr (kAdd) {
      v += bf(a.r[row * a.sr + j]);
      a.s[row * a.ss + j] = __float2bfloat16_rn(v);
    }
    srow[j] = v;
    t += kLayerNorm ? v : v * v;
  }
  const float inv_n = 1.f / static_cast<float>(n);
  float mean = 0.f;
  float stat = group_sum<kThreads>(t, red);
  if constexpr (kLayerNorm) {
    mean = stat * inv_n;
    float q = 0.f;
    for (int j = threadIdx.x; j < n; j += kThreads) {
      const float d = srow[j] - mean;
      q += d * d;
    }
    stat = group_sum<kThreads>(q, red);
  }
  const float rstd = rsqrtf(stat * inv_n + a.eps);
  for (int j = threadIdx.x; j < n; j += kThreads) {
    const float w = load_w1(a.w, a.w_dtype, j);
    float o;
    if constexpr (kLayerNorm) o = (srow[j] - mean) * rstd * w + load_w1(a.b, a.w_dtype, j);
    else o = srow[j] * rstd * w;
    if constexpr (kAxpy) o = fmaf(a.alpha, o, bf(a.base[row * a.sb + j]));
    a.y[row * a.sy + j] = __float2bfloat16_rn(o);
  }
}

template <int TPR, int VPT, bool kAdd, bool kLN, bool kAxpy>
void launch_vec(const NormArgs& a, cudaStream_t st) {
  constexpr int kRowsPerCta = kThreads / TPR;
  const int64_t grid = (a.rows + kRowsPerCta - 1) / kRowsPerCta;
  prefer_max_shared<norm_vec_kernel<TPR, VPT, kAdd, kLN, kAxpy>>();
  launch_pdl(norm_vec_kernel<TPR, VPT, kAdd, kLN, kAxpy>, dim3(static_cast<unsigned>(grid)),
             dim3(kThreads), 0, st, a);
}

template <bool kAdd, bool kLN, bool kAxpy = false>
int dispatch(const NormArgs& a, bool vec_ok, cudaStream_t st) {
  if (a.rows > 0x7fffffffLL) return fail(UMIC_ERR_UNSUPPORTED, "norm: too many rows");
  const int c = a.n >> 3;
  if (vec_ok) {
    if (c <= 4) launch_vec<4, 1, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 8) launch_vec<8, 1, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 16) launch_vec<16, 1, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 32) launch_vec<32, 1, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 64) launch_vec<32, 2, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 128) launch_vec<32, 4, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 160) launch_vec<32, 5, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 256) launch_vec<128, 2, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 512) launch_vec<256, 2, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 1024) launch_vec<256, 4, kAdd, kLN, kAxpy>(a, st);
    else if (c <= 2048) launch_vec<256, 8, kAdd, kLN, kAxpy>(a, st);
    else vec_ok = false;
  }
  if (!vec_ok) {
    if (a.n > kScalarMaxN)
      return fail(UMIC_ERR_UNSUPPORTED, "norm: n=%d exceeds %d", a.n, kScalarMaxN);
    const size_t smem = static_cast<size_t>(a.n) * sizeof(float);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(norm_scalar_kernel<kAdd, kLN, kAxpy>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    prefer_max_shared<norm_scalar_kernel<kAdd, kLN, kAxpy>>();
    norm_scalar_kernel<kAdd, kLN, kAxpy>
        <<<static_cast<unsigned>(a.rows), kThreads, smem, st>>>(a);
  }
  return launch_status("norm launch");
}

int check_common(const char* name, const void* x, const void* w, const void* y, int64_t rows,
                 int64_t n, int w_dtype) {
  if (rows < 0 || n <= 0) return fail(UMIC_ERR_INVALID_ARG, "%s: rows=%lld n=%lld", name,
                                      (long long)rows, (long long)n);
  if (rows == 0) return UMIC_OK;  // empty tensors may carry null data pointers
  if (!x || !w || !y) return fail(UMIC_ERR_INVALID_ARG, "%s: null pointer", name);
  if (n > 0x7fffffff) return fail(UMIC_ERR_UNSUPPORTED, "%s: n too large", name);
  if (w_dtype != UMIC_DTYPE_BF16 && w_dtype != UMIC_DTYPE_FP32)
    return fail(UMIC_ERR_INVALID_ARG, "%s: bad w_dtype %d", name, w_dtype);
  return UMIC_OK;
}

// The 16-byte path needs n, every row stride and every base pointer aligned.
bool vec_ok(int64_t n, std::initializer_list<const void*> ptrs,
            std::initializer_list<int64_t> strides, const void* w, int w_dtype) {
  if (n % 8) return false;
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return false;
  for (int64_t s : strides)
    if (s % 8) return false;
  if (w_dtype == UMIC_DTYPE_FP32 ? (reinterpret_cast<uintptr_t>(w) & 31u) != 0 : !aligned16(w))
    return false;
  return true;
}

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" {

int umic_rmsnorm(const void* x, int64_t sx, const void* w, int w_dtype, void* y, int64_t sy,
                 int64_t rows, int64_t n, float eps, void* stream) {
  clear_error();
  if (int rc = check_common("umic_rmsnorm", x, w, y, rows, n, w_dtype)) return rc;
  if (rows == 0) return UMIC_OK;
  NormArgs a{static_cast<const __nv_bfloat16*>(x), nullptr, w, nullptr,
             static_cast<__nv_bfloat16*>(y), nullptr, nullptr, sx, 0, sy, 0, 0, 0.f, rows,
             static_cast<int>(n), w_dtype, eps};
  return dispatch<false, false>(a, vec_ok(n, {x, y}, {sx, sy}, w, w_dtype), as_stream(stream));
}

int umic_add_rmsnorm(const void* x, int64_t sx, const void* r, int64_t sr, const void* w,
                     int w_dtype, void* normed, int64_t sn, void* summed, int64_t ss,
                     int64_t rows, int64_t n, float eps, void* stream) {
  clear_error();
  if (int rc = check_common("umic_add_rmsnorm", x, w, normed, rows, n, w_dtype)) return rc;
  if (rows == 0) return UMIC_OK;
  if (!r || !summed) return fail(UMIC_ERR_INVALID_ARG, "umic_add_rmsnorm: null pointer");
  NormArgs a{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(r), w,
             nullptr, static_cast<__nv_bfloat16*>(normed), static_cast<__nv_bfloat16*>(summed),
             nullptr, sx, sr, sn, ss, 0, 0.f, rows, static_cast<int>(n), w_dtype, eps};
  return dispatch<true, false>(
      a, vec_ok(n, {x, r, normed, summed}, {sx, sr, sn, ss}, w, w_dtype), as_stream(stream));
}

int umic_layernorm(const void* x, int64_t sx, const void* w, const void* b, int w_dtype,
                   void* y, int64_t sy, int64_t rows, int64_t n, float eps, void* stream) {
  clear_error();
  if (int rc = check_common("umic_layernorm", x, w, y, rows, n, w_dtype)) return rc;
  if (rows == 0) return UMIC_OK;
  if (!b) return fail(UMIC_ERR_INVALID_ARG, "umic_layernorm: null bias");
  NormArgs a{static_cast<const __nv_bfloat16*>(x), nullptr, w, b,
             static_cast<__nv_bfloat16*>(y), nullptr, nullptr, sx, 0, sy, 0, 0, 0.f, rows,
             static_cast<int>(n), w_dtype, eps};
  bool ok = vec_ok(n, {x, y}, {sx, sy}, w, w_dtype) && vec_ok(n, {}, {}, b, w_dtype);
  return dispatch<false, true>(a, ok, as_stream(stream));
}

int umic_add_layernorm(const void* x, int64_t sx, const void* r, int64_t sr, const void* w,
                       const void* b, int w_dtype, void* normed, int64_t sn, void* summed,
                       int64_t ss, int64_t rows, int64_t n, float eps, void* stream) {
  clear_error();
  if (int rc = check_common("umic_add_layernorm", x, w, normed, rows, n, w_dtype)) return rc;
  if (rows == 0) return UMIC_OK;
  if (!r || !summed || !b) return fail(UMIC_ERR_INVALID_ARG, "umic_add_layernorm: null pointer");
  NormArgs a{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(r), w, b,
             static_cast<__nv_bfloat16*>(normed), static_cast<__nv_bfloat16*>(summed), nullptr,
             sx, sr, sn, ss, 0, 0.f, rows, static_cast<int>(n), w_dtype, eps};
  bool ok = vec_ok(n, {x, r, normed, summed}, {sx, sr, sn, ss}, w, w_dtype) &&
            vec_ok(n, {}, {}, b, w_dtype);
  return dispatch<true, true>(a, ok, as_stream(stream));
}

int umic_rmsnorm_axpy(const void* x, int64_t sx, const void* w, int w_dtype, const void* base,
                      int64_t sb, float alpha, void* y, int64_t sy, int64_t rows, int64_t n,
                      float eps, void* stream) {
  clear_error();
  if (int rc = check_common("umic_rmsnorm_axpy", x, w, y, rows, n, w_dtype)) return rc;
  if (rows == 0) return UMIC_OK;
  if (!base) return fail(UMIC_ERR_INVALID_ARG, "umic_rmsnorm_axpy: null base");
  if (sx <= 0 || sb <= 0 || sy <= 0)
    return fail(UMIC_ERR_INVALID_ARG, "umic_rmsnorm_axpy: row strides must be positive");
  NormArgs a{static_cast<const __nv_bfloat16*>(x), nullptr, w, nullptr,
             static_cast<__nv_bfloat16*>(y), nullptr, static_cast<const __nv_bfloat16*>(base),
             sx, 0, sy, 0, sb, alpha, rows, static_cast<int>(n), w_dtype, eps};
  return dispatch<false, false, true>(a, vec_ok(n, {x, y, base}, {sx, sy, sb}, w, w_dtype),
                                      as_stream(stream));
}

}  // extern "C"
