// Decode-regime projection (rows < FUSE_MIN_ROWS): y[m, n] = x[m, :] . w[n, :].
//
// HBM-bound: every weight byte is read once, the activations (m <= 63 rows)
// stay in L1/L2. The dot products run on the tensor cores through
// mma.sync.m16n8k16 so the math costs nothing next to the weight stream:
//   - a warp owns 16 weight rows; the 8 activation rows of an m-chunk are the
//     n8 side of the MMA; m <= 63 uses up to 8 chunks that reuse the weight
//     registers;
//   - lane (g = lane/4, t = lane%4) loads w[n0+g][k+8t .. k+8t+7] and
//     w[n0+g+8][...] as two 16-byte vectors, and x[g][k+8t .. +7] as one.
//     A dot product does not depend on the order of its k terms, so the same
//     permutation of k applied to both operands lets these 16-byte loads be
//     the MMA fragments directly (two m16n8k16 steps per 32-wide k slab), with
//     no shared-memory staging and no bf16->fp32 conversions;
//   - the warps of a CTA split k into contiguous ranges and meet in shared
//     memory at the end;
//   - small matrices (k/v projections, N = 1024) would leave most SMs idle
//     with one CTA per 16 rows, so k is also split across a thread-block
//     cluster of up to 8 CTAs; their partial sums meet in the leader CTA
//     through distributed shared memory (no global scratch, no atomics).
// The gated variant streams gate and up rows together and applies
// silu(g) * u before the single bf16 rounding (fused_ffn.py:86-87 semantics).
#include <cooperative_groups.h>

#include "common.cuh"

namespace umic {
namespace {

// One weight matrix of a (possibly multi-matrix) launch: rows [row0, row0 + rows)
// of the concatenated row space are rows [0, rows) of w, written to y.
struct Seg {
  const __nv_bfloat16* w;
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;
  int64_t ldw, ldy;
  int row0, rows;
};

constexpr int kMaxSeg = 3;

struct GemvArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w2;  // up weights of the gated variant (segment 0 holds gate)
  int64_t ldx;
  Seg seg[kMaxSeg];
  int nseg;
  int m, n, k;  // n = total rows over the segments
  int slabs;    // ceil(k / 32)
};

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two k16 steps from one 32-wide slab: rows g / g+8 of w (wlo / whi) and
// row g of x, each 8 consecutive k values held as a uint4.
__device__ __forceinline__ void slab_mma(float (&c)[4], const uint4& wlo, const uint4& whi,
                                         const uint4& xv) {
  mma16816(c, wlo.x, whi.x, wlo.y, whi.y, xv.x, xv.y);
  mma16816(c, wlo.z, whi.z, wlo.w, whi.w, xv.z, xv.w);
}

namespace cg = cooperative_groups;

template <int MC, bool kGated>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  // Weight slabs loaded before any math: 8 for the plain small-M case (2 KB of
  // loads in flight per lane-group of the warp), 4 when registers are scarcer.
  constexpr int kUnroll = (!kGated && MC <= 2) ? 8 : 4;
  // [warps][kGated+1][MC][4][32] per-warp fragments, then [kGated+1][MC][4][32]
  // CTA totals (read by the cluster leader).
  extern __shared__ float red[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int csplit = gridDim.y, crank = blockIdx.y;  // k split across the cluster
  // The segment this CTA's 16 rows belong to (boundaries are multiples of 16).
  int si = 0;
  while (si + 1 < a.nseg && static_cast<int>(blockIdx.x) * 16 >= a.seg[si + 1].row0) ++si;
  const Seg sg = a.seg[si];
  const int n0 = blockIdx.x * 16 - sg.row0;  // first row inside the segment
  const int r0 = n0 + g, r1 = n0 + g + 8;
  const bool r0ok = r0 < sg.rows, r1ok = r1 < sg.rows;
  const __nv_bfloat16* wp = sg.w;

  float acc[MC][4];
  float acc2[kGated ? MC : 1][4];
#pragma unroll
  for (int i = 0; i < MC; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[i][j] = 0.f;
      if constexpr (kGated) acc2[i][j] = 0.f;
    }

  // Contiguous slab range of this CTA, then of this warp.
  const int per_cta = (a.slabs + csplit - 1) / csplit;
  const int c_begin = crank * per_cta;
  const int c_end = min(a.slabs, c_begin + per_cta);
  const int per = (c_end - c_begin + nwarps - 1) / nwarps;
  const int s_begin = c_begin + warp * per;
  const int s_end = min(c_end, s_begin + per);
  const uint4 zero = make_uint4(0, 0, 0, 0);

  for (int s0 = s_begin; s0 < s_end; s0 += kUnroll) {
    uint4 wl[kUnroll], wh[kUnroll], ul[kGated ? kUnroll : 1], uh[kGated ? kUnroll : 1];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int kk = (s0 + u) * 32 + t * 8;
      const bool kok = (s0 + u) < s_end && kk < a.k;
      wl[u] = (kok && r0ok) ? ld_stream(wp + r0 * sg.ldw + kk) : zero;
      wh[u] = (kok && r1ok) ? ld_stream(wp + r1 * sg.ldw + kk) : zero;
      if constexpr (kGated) {
        ul[u] = (kok && r0ok) ? ld_stream(a.w2 + r0 * sg.ldw + kk) : zero;
        uh[u] = (kok && r1ok) ? ld_stream(a.w2 + r1 * sg.ldw + kk) : zero;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int kk = (s0 + u) * 32 + t * 8;
      const bool kok = (s0 + u) < s_end && kk < a.k;
#pragma unroll
      for (int mc = 0; mc < MC; ++mc) {
        const int xr = mc * 8 + g;
        const uint4 xv = (kok && xr < a.m) ? ld_cached(a.x + xr * a.ldx + kk) : zero;
        slab_mma(acc[mc], wl[u], wh[u], xv);
        if constexpr (kGated) slab_mma(acc2[mc], ul[u], uh[u], xv);
      }
    }
  }

  // Cross-warp reduction of the C fragments.
  constexpr int kAcc = kGated ? 2 : 1;
  float* mine = red + static_cast<size_t>(warp) * kAcc * MC * 4 * 32;
#pragma unroll
  for (int mc = 0; mc < MC; ++mc)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mine[(mc * 4 + j) * 32 + lane] = acc[mc][j];
      if constexpr (kGated) mine[((MC + mc) * 4 + j) * 32 + lane] = acc2[mc][j];
    }
  __syncthreads();
  const int stride = kAcc * MC * 4 * 32;
  float* tot = red + static_cast<size_t>(nwarps) * stride;  // CTA totals
  for (int i = threadIdx.x; i < stride; i += blockDim.x) {
    float v = 0.f;
    for (int w = 0; w < nwarps; ++w) v += red[w * stride + i];
    tot[i] = v;
  }
  if (csplit > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every CTA's totals are in its shared memory
    if (crank == 0 && warp == 0) {
      for (int r = 1; r < csplit; ++r) {
        const float* remote = cluster.map_shared_rank(tot, r);
        for (int i = lane; i < stride; i += 32) tot[i] += remote[i];
      }
    }
    cluster.sync();  // the leader has read them; peers may exit
    if (crank != 0) return;
  } else {
    __syncthreads();
  }
  if (warp != 0) return;
#pragma unroll
  for (int mc = 0; mc < MC; ++mc) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v = tot[(mc * 4 + j) * 32 + lane];
      const float v2 = kGated ? tot[((MC + mc) * 4 + j) * 32 + lane] : 0.f;
      // C fragment: c0,c1 -> (row g, cols 2t,2t+1); c2,c3 -> (row g+8, ...)
      const int nrow = (j < 2) ? r0 : r1;
      const int mcol = mc * 8 + 2 * t + (j & 1);
      if (nrow >= sg.rows || mcol >= a.m) continue;
      float o;
      if constexpr (kGated) {
        o = v / (1.f + __expf(-v)) * v2;
      } else {
        o = v;
        if (sg.bias) o += bf(sg.bias[nrow]);
      }
      sg.y[mcol * sg.ldy + nrow] = __float2bfloat16_rn(o);
    }
  }
}

template <int MC, bool kGated>
int launch(const GemvArgs& a, cudaStream_t st) {
  const int row_blocks = (a.n + 15) / 16;
  // Aim for about 4 CTAs per SM; split k over a cluster when the rows alone
  // give fewer, while keeping at least 4 slabs of 32 per CTA.
  // 4-warp CTAs, about 6 resident per SM: 768 row blocks (a 12288-row matrix)
  // then fill one wave on 148 SMs instead of spilling a few CTAs into a second
  // wave. Matrices with fewer row blocks split k across a cluster (up to 8 CTAs,
  // keeping at least 8 slabs of 32 per CTA).
  const int target = 5 * sm_count();
  int csplit = 1;
  while (csplit < 8 && row_blocks * csplit < target && a.slabs / (csplit * 2) >= 8) csplit *= 2;
  const int warps = 4;
  const size_t smem =
      static_cast<size_t>(warps + 1) * (kGated ? 2 : 1) * MC * 4 * 32 * sizeof(float);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(gemv_kernel<MC, kGated>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(row_blocks, csplit, 1);
  cfg.blockDim = dim3(warps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = csplit;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_kernel<MC, kGated>, a);
  if (e != cudaSuccess) return fail(UMIC_ERR_LAUNCH, "umic_gemv launch: %s", cudaGetErrorString(e));
  return launch_status("umic_gemv launch");
}

template <bool kGated>
int dispatch(const GemvArgs& a, cudaStream_t st) {
  switch ((a.m + 7) / 8) {
    case 1: return launch<1, kGated>(a, st);
    case 2: return launch<2, kGated>(a, st);
    case 3: return launch<3, kGated>(a, st);
    case 4: return launch<4, kGated>(a, st);
    case 5: return launch<5, kGated>(a, st);
    case 6: return launch<6, kGated>(a, st);
    case 7: return launch<7, kGated>(a, st);
    case 8: return launch<8, kGated>(a, st);
  }
  return fail(UMIC_ERR_UNSUPPORTED, "umic_gemv: m=%d outside 1..64", a.m);
}

int check(const char* name, const void* x, int64_t ldx, const void* w, const void* w2,
          int64_t ldw, const void* y, int64_t ldy, int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k <= 0) return fail(UMIC_ERR_INVALID_ARG, "%s: bad sizes", name);
  if (m == 0 || n == 0) return UMIC_OK;
  if (!x || !w || !w2 || !y) return fail(UMIC_ERR_INVALID_ARG, "%s: null pointer", name);
  if (m > 64) return fail(UMIC_ERR_UNSUPPORTED, "%s: m=%lld > 64 (use umic_gemm)", name,
                          (long long)m);
  if (n > 0x7fffffffLL - 16 || k > 0x7fffffffLL - 64)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: n or k too large", name);
  if (k % 8 || ldx % 8 || ldw % 8 || !aligned16(x) || !aligned16(w) || !aligned16(w2))
    return fail(UMIC_ERR_ALIGNMENT, "%s: k, ldx, ldw must be multiples of 8 and x, w 16-byte "
                "aligned", name);
  if (ldx < k || ldw < k || ldy < n) return fail(UMIC_ERR_INVALID_ARG, "%s: leading dim", name);
  return UMIC_OK;
}

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" {

int umic_gemv(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias, void* y,
              int64_t ldy, int64_t m, int64_t n, int64_t k, void* stream) {
  clear_error();
  if (int rc = check("umic_gemv", x, ldx, w, w, ldw, y, ldy, m, n, k)) return rc;
  if (m == 0 || n == 0) return UMIC_OK;  // nothing to launch
  GemvArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.seg[0] = Seg{static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(bias),
                 static_cast<__nv_bfloat16*>(y), ldw, ldy, 0, static_cast<int>(n)};
  a.nseg = 1;
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  a.slabs = static_cast<int>((k + 31) / 32);
  return dispatch<false>(a, as_stream(stream));
}

int umic_gemv_multi(const void* x, int64_t ldx, int32_t count, const void* const* w,
                    const int64_t* ldw, const int64_t* n, const void* const* bias,
                    void* const* y, const int64_t* ldy, int64_t m, int64_t k, void* stream) {
  clear_error();
  if (count < 1 || count > kMaxSeg || !w || !ldw || !n || !y || !ldy)
    return fail(UMIC_ERR_INVALID_ARG, "umic_gemv_multi: count=%d or null array", count);
  GemvArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  int64_t total = 0;
  for (int i = 0; i < count; ++i) {
    if (int rc = check("umic_gemv_multi", x, ldx, w[i], w[i], ldw[i], y[i], ldy[i], m, n[i], k))
      return rc;
    if (n[i] <= 0) return fail(UMIC_ERR_INVALID_ARG, "umic_gemv_multi: empty matrix %d", i);
    if (i + 1 < count && n[i] % 16)
      return fail(UMIC_ERR_UNSUPPORTED, "umic_gemv_multi: rows of matrix %d not a multiple of 16",
                  i);
    a.seg[i] = Seg{static_cast<const __nv_bfloat16*>(w[i]),
                   bias ? static_cast<const __nv_bfloat16*>(bias[i]) : nullptr,
                   static_cast<__nv_bfloat16*>(y[i]), ldw[i], ldy[i], static_cast<int>(total),
                   static_cast<int>(n[i])};
    total += n[i];
  }
  if (m == 0) return UMIC_OK;
  if (total > 0x7fffffffLL - 16) return fail(UMIC_ERR_UNSUPPORTED, "umic_gemv_multi: too many rows");
  a.nseg = count;
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(total);
  a.k = static_cast<int>(k);
  a.slabs = static_cast<int>((k + 31) / 32);
  return dispatch<false>(a, as_stream(stream));
}

int umic_gemv_gate_silu_mul(const void* x, int64_t ldx, const void* wg, const void* wu,
                            int64_t ldw, void* h, int64_t ldh, int64_t m, int64_t n, int64_t k,
                            void* stream) {
  clear_error();
  if (int rc = check("umic_gemv_gate_silu_mul", x, ldx, wg, wu, ldw, h, ldh, m, n, k)) return rc;
  if (m == 0 || n == 0) return UMIC_OK;
  GemvArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.w2 = static_cast<const __nv_bfloat16*>(wu);
  a.ldx = ldx;
  a.seg[0] = Seg{static_cast<const __nv_bfloat16*>(wg), nullptr, static_cast<__nv_bfloat16*>(h),
                 ldw, ldh, 0, static_cast<int>(n)};
  a.nseg = 1;
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  a.slabs = static_cast<int>((k + 31) / 32);
  return dispatch<true>(a, as_stream(stream));
}

}  // extern "C"
