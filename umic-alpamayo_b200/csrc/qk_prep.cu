// Attention input preparation in one pass: per-head RMSNorm of q and k, rotate-half
// RoPE of both, and the K/V write into the in-place cache.
//
// The reference runs this as separate steps -- q_norm and k_norm (one RMSNorm
// launch each, src/umic/integrate.py:134-141 applied to the per-head norms),
// apply_rotary_pos_emb (src/umic/kernels/rope.py:86-107) and the cache write
// (src/umic/cache.py:59-60, 69-70) -- each reading and writing q/k through HBM.
// Here a group of D/8 threads owns one head row of one token (8 consecutive
// elements per thread, 16-byte loads): the sum of squares is reduced with
// shuffles inside the group, the normalised values stay in registers, and the
// RoPE partner (element d +/- D/2) is held by the thread D/16 lanes away, so one
// shuffle brings it over. q is written back in place; k (normalised, rotated)
// and v (copied) go straight to [b, h, pos + s, :] of the cache buffers, or k is
// written back in place when no cache buffer is given. Math in fp32, one bf16
// rounding per output.
#include "common.cuh"

namespace umic {
namespace {

struct PrepArgs {
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const void* qw;
  const void* kw;
  const void* cos;
  const void* sin;
  __nv_bfloat16* kb;
  __nv_bfloat16* vb;
  const int64_t* dpos;
  uint32_t* err;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  int64_t v_sb, v_ss, v_sh;
  int64_t c_sb, c_ss;
  int64_t b_sb, b_sh, b_ss;
  int64_t capacity;
  int64_t pos;
  int64_t seq;
  int hq, hk;
  int w_dtype;
  int cos_fp32;
  float q_eps, k_eps;
};

__device__ __forceinline__ void load_table8(const void* base, bool fp32, int64_t idx,
                                            float (&f)[8]) {
  if (fp32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    unpack8(ld_cached(static_cast<const __nv_bfloat16*>(base) + idx), f);
  }
}

// block = 256 threads = 256 / TPH head rows of one token; grid = (seq, batch,
// ceil(rows / rows per block)). Row index r: [0, hq) q heads, [hq, hq+hk) k heads,
// then [hq+hk, hq+2hk) v heads when the K/V go to a cache.
template <int TPH>
__global__ void __launch_bounds__(256) qk_prep_kernel(PrepArgs a) {
  constexpr int kRowsPerBlock = 256 / TPH;
  constexpr int kHalf = TPH / 2;  // partner lane distance (D/16 threads)
  const int sub = threadIdx.x % TPH;
  const int r = blockIdx.z * kRowsPerBlock + threadIdx.x / TPH;
  const int64_t s = blockIdx.x, b = blockIdx.y;
  const int rows = a.hq + (a.kb ? 2 * a.hk : a.hk);  // v rows only with a cache write
  const bool active = r < rows;
  int64_t pos = 0;
  if (a.kb) {
    pos = a.dpos ? *a.dpos : a.pos;
    if (pos < 0 || pos + a.seq > a.capacity) {
      if (threadIdx.x == 0 && s == 0 && b == 0 && blockIdx.z == 0 && a.err)
        atomicOr(a.err, UMIC_DEVERR_KV_OVERFLOW);
      return;  // uniform for the whole grid
    }
  }
  const int d0 = sub * 8;
  float x[8];
  // v rows: plain copy into the cache (no norm, no rotation)
  const bool is_v = active && r >= a.hq + a.hk;
  if (is_v) {
    const int h = r - a.hq - a.hk;
    const uint4 val = ld_stream(a.v + b * a.v_sb + s * a.v_ss + h * a.v_sh + d0);
    if (a.kb) st_vec(a.vb + b * a.b_sb + h * a.b_sh + (pos + s) * a.b_ss + d0, val);
  }
  const bool is_q = active && r < a.hq;
  const bool is_k = active && !is_q && !is_v;
  __nv_bfloat16* src = nullptr;
  if (is_q) src = a.q + b * a.q_sb + s * a.q_ss + r * a.q_sh;
  else if (is_k) src = a.k + b * a.k_sb + s * a.k_ss + (r - a.hq) * a.k_sh;
  if (src) unpack8(ld_stream(src + d0), x);
  else {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = 0.f;
  }
  // per-head RMSNorm (all lanes of the group take part in the shuffles)
  const void* w = is_q ? a.qw : a.kw;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
#pragma unroll
  for (int o = TPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (w && src) {
    const float rstd = rsqrtf(ss / static_cast<float>(TPH * 8) + (is_q ? a.q_eps : a.k_eps));
    float wv[8];
    load_w8(w, a.w_dtype, d0, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = x[j] * rstd * wv[j];
  }
  // rotate-half RoPE: lanes sub < kHalf hold the first half, their partners sub + kHalf
  float p[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) p[j] = __shfl_xor_sync(0xffffffffu, x[j], kHalf);
  if (!src) return;
  const int64_t crow = b * a.c_sb + s * a.c_ss;
  float c[8], sn[8];
  load_table8(a.cos, a.cos_fp32, crow + d0, c);
  load_table8(a.sin, a.cos_fp32, crow + d0, sn);
  float o[8];
  if (sub < kHalf) {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = x[j] * c[j] - p[j] * sn[j];
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = x[j] * c[j] + p[j] * sn[j];
  }
  const uint4 out = pack8(o);
  if (is_q || !a.kb) {
    st_vec(src + d0, out);
  } else {
    const int h = r - a.hq;
    st_vec(a.kb + b * a.b_sb + h * a.b_sh + (pos + s) * a.b_ss + d0, out);
  }
}

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" int umic_qk_norm_rope_kv(
    void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, int32_t hq, void* k, int64_t k_sb,
    int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
    int32_t hk, const void* q_weight, const void* k_weight, int w_dtype, float q_eps,
    float k_eps, const void* cos, const void* sin, int64_t c_sb, int64_t c_ss, int cos_dtype,
    void* k_buf, void* v_buf, int64_t buf_sb, int64_t buf_sh, int64_t buf_ss, int64_t capacity,
    int64_t pos, const int64_t* dpos, int64_t batch, int64_t seq, int32_t head_dim,
    void* stream) {
  clear_error();
  if (hq <= 0 || hk <= 0 || batch < 0 || seq < 0)
    return fail(UMIC_ERR_INVALID_ARG, "umic_qk_norm_rope_kv: hq=%d hk=%d", hq, hk);
  if (batch == 0 || seq == 0) return UMIC_OK;
  if (!q || !k || !cos || !sin || (k_buf && (!v || !v_buf)))
    return fail(UMIC_ERR_INVALID_ARG, "umic_qk_norm_rope_kv: null pointer");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(UMIC_ERR_UNSUPPORTED, "umic_qk_norm_rope_kv: head_dim %d (64, 128 or 256)",
                head_dim);
  if (w_dtype != UMIC_DTYPE_BF16 && w_dtype != UMIC_DTYPE_FP32)
    return fail(UMIC_ERR_INVALID_ARG, "umic_qk_norm_rope_kv: bad w_dtype");
  if (cos_dtype != UMIC_DTYPE_BF16 && cos_dtype != UMIC_DTYPE_FP32)
    return fail(UMIC_ERR_INVALID_ARG, "umic_qk_norm_rope_kv: bad cos_dtype");
  const int64_t celem = cos_dtype == UMIC_DTYPE_FP32 ? 4 : 8;
  const bool aligned = aligned16(q) && aligned16(k) && aligned16(cos) && aligned16(sin) &&
                       (!v || aligned16(v)) && (!k_buf || (aligned16(k_buf) && aligned16(v_buf))) &&
                       q_sb % 8 == 0 && q_ss % 8 == 0 && q_sh % 8 == 0 && k_sb % 8 == 0 &&
                       k_ss % 8 == 0 && k_sh % 8 == 0 && v_sb % 8 == 0 && v_ss % 8 == 0 &&
                       v_sh % 8 == 0 && buf_sb % 8 == 0 && buf_sh % 8 == 0 &&
                       buf_ss % 8 == 0 && c_sb % celem == 0 && c_ss % celem == 0;
  if (!aligned)
    return fail(UMIC_ERR_ALIGNMENT, "umic_qk_norm_rope_kv: 16-byte alignment of bases/strides");
  const bool wq_al = !q_weight || (w_dtype == UMIC_DTYPE_FP32
                                       ? (reinterpret_cast<uintptr_t>(q_weight) & 31u) == 0
                                       : aligned16(q_weight));
  const bool wk_al = !k_weight || (w_dtype == UMIC_DTYPE_FP32
                                       ? (reinterpret_cast<uintptr_t>(k_weight) & 31u) == 0
                                       : aligned16(k_weight));
  if (!wq_al || !wk_al) return fail(UMIC_ERR_ALIGNMENT, "umic_qk_norm_rope_kv: norm weights");
  if (k_buf && !dpos && (pos < 0 || pos + seq > capacity))
    return fail(UMIC_ERR_OVERFLOW, "InplaceLayer overflow: pos %lld + new %lld > buffer %lld",
                (long long)pos, (long long)seq, (long long)capacity);
  if (batch > 65535 || seq > 0x7fffffffLL)
    return fail(UMIC_ERR_UNSUPPORTED, "umic_qk_norm_rope_kv: batch/seq too large");
  PrepArgs a{static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k),
             static_cast<const __nv_bfloat16*>(v), q_weight, k_weight, cos, sin,
             static_cast<__nv_bfloat16*>(k_buf), static_cast<__nv_bfloat16*>(v_buf), dpos,
             device_error_word(), q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, v_sb, v_ss, v_sh, c_sb,
             c_ss, buf_sb, buf_sh, buf_ss, capacity, pos, seq, hq, hk, w_dtype,
             cos_dtype == UMIC_DTYPE_FP32 ? 1 : 0, q_eps, k_eps};
  const int tph = head_dim / 8;
  const int rows_per_block = 256 / tph;
  const int rows = hq + (k_buf ? 2 * hk : hk);
  const dim3 grid(static_cast<unsigned>(seq), static_cast<unsigned>(batch),
                  static_cast<unsigned>((rows + rows_per_block - 1) / rows_per_block));
  cudaStream_t st = as_stream(stream);
  if (tph == 8) qk_prep_kernel<8><<<grid, 256, 0, st>>>(a);
  else if (tph == 16) qk_prep_kernel<16><<<grid, 256, 0, st>>>(a);
  else qk_prep_kernel<32><<<grid, 256, 0, st>>>(a);
  return launch_status("umic_qk_norm_rope_kv");
}
