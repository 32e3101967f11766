// In-place rotate-half RoPE for q and k in one launch.
//
// A thread owns one 8-element slice of the first half of a head row plus the
// matching slice of the second half, so it holds both members of every
// rotation pair and no partner gather is needed (the reference gathers the
// partner by index, rope.py:49-52). A block covers all heads of q and k at a
// few positions: the cos/sin row of a position is fetched from DRAM once and
// served from L1 to every head. The 3-D block shape (slice, head, position)
// makes the index arithmetic division-free.
//   text   D=128: 8 items per head row, cos/sin bf16 [B,S,128]
//   vision D=80 : 5 items per head row, cos/sin fp32 [S,80], q/k rows 3840 apart
// Math in fp32 with one rounding to bf16 (rope.py:45-60).
#include "common.cuh"

namespace umic {
namespace {

struct RopeArgs {
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  const void* cos;
  const void* sin;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  int64_t c_sb, c_ss;
  int64_t seq;
  int hq, hk;
  int half;
};

__device__ __forceinline__ void load_cs8(const void* base, bool fp32, int64_t idx,
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

__device__ __forceinline__ float load_cs1(const void* base, bool fp32, int64_t idx) {
  return fp32 ? __ldg(static_cast<const float*>(base) + idx)
              : bf(static_cast<const __nv_bfloat16*>(base)[idx]);
}

// Thread (x, y, z) of block (bx, by, bz) handles slice x of head
// bz*blockDim.y + y at position bx*blockDim.z + z of batch row by, so no
// index division is needed. Returns nullptr when outside the tensor.
__device__ __forceinline__ __nv_bfloat16* locate(const RopeArgs& a, int64_t& crow) {
  const int64_t s = static_cast<int64_t>(blockIdx.x) * blockDim.z + threadIdx.z;
  const int h = blockIdx.z * blockDim.y + threadIdx.y;
  if (s >= a.seq || h >= a.hq + a.hk) return nullptr;
  const int64_t b = blockIdx.y;
  crow = b * a.c_sb + s * a.c_ss;
  if (h < a.hq) return a.q + b * a.q_sb + s * a.q_ss + h * a.q_sh;
  return a.k + b * a.k_sb + s * a.k_ss + (h - a.hq) * a.k_sh;
}

template <bool kCosFp32>
__global__ void __launch_bounds__(1024) rope_vec_kernel(RopeArgs a) {
  allow_dependent_launch();
  wait_prerequisite();
  int64_t crow;
  __nv_bfloat16* row = locate(a, crow);
  if (!row) return;
  const int d0 = threadIdx.x * 8;
  float x1[8], x2[8], c1[8], c2[8], s1[8], s2[8];
  unpack8(ld_stream(row + d0), x1);
  unpack8(ld_stream(row + a.half + d0), x2);
  load_cs8(a.cos, kCosFp32, crow + d0, c1);
  load_cs8(a.cos, kCosFp32, crow + a.half + d0, c2);
  load_cs8(a.sin, kCosFp32, crow + d0, s1);
  load_cs8(a.sin, kCosFp32, crow + a.half + d0, s2);
  float o1[8], o2[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    o1[j] = x1[j] * c1[j] - x2[j] * s1[j];
    o2[j] = x2[j] * c2[j] + x1[j] * s2[j];
  }
  st_vec(row + d0, pack8(o1));
  st_vec(row + a.half + d0, pack8(o2));
}

// Any even head_dim / alignment: one rotation pair per thread.
__global__ void __launch_bounds__(1024) rope_scalar_kernel(RopeArgs a, bool cos_fp32) {
  allow_dependent_launch();
  wait_prerequisite();
  int64_t crow;
  __nv_bfloat16* row = locate(a, crow);
  if (!row) return;
  for (int d = threadIdx.x; d < a.half; d += blockDim.x) {
    const float x1 = bf(row[d]), x2 = bf(row[d + a.half]);
    const float o1 = x1 * load_cs1(a.cos, cos_fp32, crow + d) -
                     x2 * load_cs1(a.sin, cos_fp32, crow + d);
    const float o2 = x2 * load_cs1(a.cos, cos_fp32, crow + a.half + d) +
                     x1 * load_cs1(a.sin, cos_fp32, crow + a.half + d);
    row[d] = __float2bfloat16_rn(o1);
    row[d + a.half] = __float2bfloat16_rn(o2);
  }
}

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" int umic_rope_inplace(void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, int32_t hq,
                                 void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh, int32_t hk,
                                 const void* cos, const void* sin, int64_t c_sb, int64_t c_ss,
                                 int cos_dtype, int64_t batch, int64_t seq, int32_t head_dim,
                                 void* stream) {
  clear_error();
  if (hq <= 0 || hk < 0 || batch < 0 || seq < 0 || head_dim <= 0 || (head_dim & 1))
    return fail(UMIC_ERR_INVALID_ARG, "umic_rope_inplace: hq=%d hk=%d head_dim=%d", hq, hk,
                head_dim);
  if (batch == 0 || seq == 0) return UMIC_OK;
  if (!q || !cos || !sin || (hk > 0 && !k))
    return fail(UMIC_ERR_INVALID_ARG, "umic_rope_inplace: null pointer");
  if (cos_dtype != UMIC_DTYPE_BF16 && cos_dtype != UMIC_DTYPE_FP32)
    return fail(UMIC_ERR_INVALID_ARG, "umic_rope_inplace: bad cos_dtype %d", cos_dtype);
  if (batch == 0 || seq == 0) return UMIC_OK;
  const bool fp32 = cos_dtype == UMIC_DTYPE_FP32;
  const int half = head_dim / 2;
  // Vector path: 8-element slices of both halves start on 16-byte boundaries
  // in q, k and the cos/sin tables.
  const int64_t celem = fp32 ? 4 : 8;  // elements per 16 bytes of cos/sin
  bool vec = (half % 8 == 0) && aligned16(q) && (!k || aligned16(k)) && aligned16(cos) &&
             aligned16(sin) && q_sb % 8 == 0 && q_ss % 8 == 0 && q_sh % 8 == 0 &&
             k_sb % 8 == 0 && k_ss % 8 == 0 && k_sh % 8 == 0 && c_sb % celem == 0 &&
             c_ss % celem == 0;
  if (batch > 65535) return fail(UMIC_ERR_UNSUPPORTED, "umic_rope_inplace: batch > 65535");
  RopeArgs a{static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), cos, sin,
             q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, c_sb, c_ss, seq, hq, hk, half};
  // Block = (slices per head row, heads, positions): about 256 threads.
  const int heads = hq + hk;
  const int bx = vec ? half / 8 : (half < 64 ? half : 64);
  const int by = heads < 1024 / bx ? heads : 1024 / bx;
  int bz = 256 / (bx * by);
  if (bz < 1) bz = 1;
  if (bz > 64) bz = 64;  // blockDim.z limit
  const dim3 block(bx, by, bz);
  const int64_t gx = (seq + bz - 1) / bz;
  if (gx > 0x7fffffffLL) return fail(UMIC_ERR_UNSUPPORTED, "umic_rope_inplace: seq too long");
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(batch),
                  static_cast<unsigned>((heads + by - 1) / by));
  cudaStream_t st = as_stream(stream);
  if (vec) {
    if (fp32) launch_pdl(rope_vec_kernel<true>, grid, block, 0, st, a);
    else launch_pdl(rope_vec_kernel<false>, grid, block, 0, st, a);
  } else {
    launch_pdl(rope_scalar_kernel, grid, block, 0, st, a, fp32);
  }
  return launch_status("umic_rope_inplace");
}
