// In-place KV-cache append: copies n_new tokens of K and V into preallocated
// [batch, heads, capacity, head_dim] buffers at a token position.
//
// The position is either a host value (checked against capacity before the
// launch) or a device int64 read when the kernel runs, which is what lets one
// captured CUDA graph per KV length replay while the position advances
// (the reference uses index_copy_ with a device index for that, cache.py:59-60).
// A device position out of range skips the write and sets
// UMIC_DEVERR_KV_OVERFLOW in the library's device error word.
// Pure copy, HBM-bound: 2 * batch * heads * n_new * head_dim * 2 bytes each way.
#include "common.cuh"

namespace umic {
namespace {

struct KvArgs {
  __nv_bfloat16* kb;
  __nv_bfloat16* vb;
  const __nv_bfloat16* kn;
  const __nv_bfloat16* vn;
  int64_t b_sb, b_sh, b_ss;
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int64_t capacity;
  int64_t n_new;
  int64_t pos;
  const int64_t* dpos;
  uint32_t* err;
  int heads;
  int head_dim;
  int chunks;  // 16-byte slices per head row (vector path) or head_dim (scalar)
};

__device__ __forceinline__ bool resolve_pos(const KvArgs& a, int64_t& pos) {
  pos = a.dpos ? *a.dpos : a.pos;
  if (pos < 0 || pos + a.n_new > a.capacity) {
    if (threadIdx.x == 0 && threadIdx.y == 0 && blockIdx.x == 0 && blockIdx.y == 0 &&
        blockIdx.z == 0 && a.err)
      atomicOr(a.err, UMIC_DEVERR_KV_OVERFLOW);
    return false;
  }
  return true;
}

// grid = (token tiles, heads, batch); block = (chunks, tokens per block).
template <bool kVec>
__global__ void __launch_bounds__(256) kv_append_kernel(KvArgs a) {
  allow_dependent_launch();
  wait_prerequisite();
  int64_t pos;
  if (!resolve_pos(a, pos)) return;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  if (t >= a.n_new) return;
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int64_t dst = b * a.b_sb + h * a.b_sh + (pos + t) * a.b_ss;
  const int64_t ks = b * a.k_sb + h * a.k_sh + t * a.k_ss;
  const int64_t vs = b * a.v_sb + h * a.v_sh + t * a.v_ss;
  if constexpr (kVec) {
    const int d = threadIdx.x * 8;
    st_vec(a.kb + dst + d, ld_stream(a.kn + ks + d));
    st_vec(a.vb + dst + d, ld_stream(a.vn + vs + d));
  } else {
    for (int d = threadIdx.x; d < a.head_dim; d += blockDim.x) {
      a.kb[dst + d] = a.kn[ks + d];
      a.vb[dst + d] = a.vn[vs + d];
    }
  }
}

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" int umic_kv_append(void* k_buf, void* v_buf, int64_t buf_sb, int64_t buf_sh,
                              int64_t buf_ss, int64_t capacity, const void* k_new, int64_t kn_sb,
                              int64_t kn_sh, int64_t kn_ss, const void* v_new, int64_t vn_sb,
                              int64_t vn_sh, int64_t vn_ss, int64_t batch, int32_t heads,
                              int64_t n_new, int32_t head_dim, int64_t pos, const int64_t* dpos,
                              void* stream) {
  clear_error();
  if (batch < 0 || heads <= 0 || n_new < 0 || head_dim <= 0 || capacity < 0)
    return fail(UMIC_ERR_INVALID_ARG, "umic_kv_append: bad sizes");
  if (batch == 0 || n_new == 0) return UMIC_OK;
  if (!k_buf || !v_buf || !k_new || !v_new)
    return fail(UMIC_ERR_INVALID_ARG, "umic_kv_append: null pointer");
  if (!dpos && (pos < 0 || pos + n_new > capacity))
    return fail(UMIC_ERR_OVERFLOW, "InplaceLayer overflow: pos %lld + new %lld > buffer %lld",
                (long long)pos, (long long)n_new, (long long)capacity);
  if (batch > 65535 || heads > 65535)
    return fail(UMIC_ERR_UNSUPPORTED, "umic_kv_append: batch/heads > 65535");
  const bool vec = head_dim % 8 == 0 && aligned16(k_buf) && aligned16(v_buf) &&
                   aligned16(k_new) && aligned16(v_new) && buf_sb % 8 == 0 &&
                   buf_sh % 8 == 0 && buf_ss % 8 == 0 && kn_sb % 8 == 0 && kn_sh % 8 == 0 &&
                   kn_ss % 8 == 0 && vn_sb % 8 == 0 && vn_sh % 8 == 0 && vn_ss % 8 == 0 &&
                   head_dim / 8 <= 256;
  KvArgs a{static_cast<__nv_bfloat16*>(k_buf), static_cast<__nv_bfloat16*>(v_buf),
           static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new),
           buf_sb, buf_sh, buf_ss, kn_sb, kn_sh, kn_ss, vn_sb, vn_sh, vn_ss, capacity, n_new,
           pos, dpos, device_error_word(), heads, head_dim, 0};
  const int bx = vec ? head_dim / 8 : (head_dim < 128 ? head_dim : 128);
  int by = 256 / bx;
  if (by < 1) by = 1;
  if (by > n_new) by = static_cast<int>(n_new);
  const int64_t gx = (n_new + by - 1) / by;
  if (gx > 0x7fffffffLL) return fail(UMIC_ERR_UNSUPPORTED, "umic_kv_append: too many tokens");
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(heads),
                  static_cast<unsigned>(batch));
  const dim3 block(bx, by);
  cudaStream_t st = as_stream(stream);
  if (vec) launch_pdl(kv_append_kernel<true>, grid, block, 0, st, a);
  else launch_pdl(kv_append_kernel<false>, grid, block, 0, st, a);
  return launch_status("umic_kv_append");
}
