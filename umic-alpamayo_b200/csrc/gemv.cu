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

#include <mutex>

#include "common.cuh"
#include "mma_frag.cuh"
#include "tma.cuh"

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

namespace cg = cooperative_groups;

template <int MC, bool kGated>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  allow_dependent_launch();
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

// =================================================================== streaming
//
// Decode rows (m <= 16) with a caller-owned workspace take this engine. The weight
// stream, which is all that matters at HBM speed, is moved by TMA instead of by the
// math warps:
//   - one persistent CTA per SM; the weight rows are cut into 64-row blocks and each
//     block into k chunks (256 columns, 128 for gate+up), a "unit" of 32 KB;
//   - the units are dealt to the CTAs as contiguous, equal ranges (stream-K), so
//     every SM streams the same number of bytes whatever the matrix shape;
//   - a producer warp keeps a 4-stage ring of units in flight (2D TMA loads with
//     128-byte swizzle, 128 KB per SM); four consumer warps read their 16 rows of
//     each unit from shared memory as the same permuted-k mma.sync fragments as the
//     cluster engine above, with x (tiny, L1/L2 resident) from global memory;
//   - a row block split between CTAs meets in the workspace: each contributor
//     stores its fp32 partial in its own slot and counts itself in with an
//     acq_rel atomic; the last one sums the slots in CTA order (deterministic),
//     writes y and resets the counter to zero for the next call;
//   - launched with programmatic stream serialization: CTA launch and barrier
//     setup overlap the end of the previous kernel in the stream; the consumers
//     wait for that kernel (griddepcontrol.wait) before touching x, y or the
//     workspace. With UMIC_GEMV_WEIGHTS_READY the producer starts streaming the
//     weights before the wait, i.e. while the previous kernel is still running;
//     without it the producer waits too.
constexpr int kStRows = 64;
// Four 32 KB stages (128 KB in flight per SM) saturate HBM and leave ~99 KB of the
// unified L1 for x, which every unit re-reads (64 KB at m = 8, k = 4096): six stages
// measured 10 % slower on lm_head and 1.2 % slower over a decode step's GEMV chain.
constexpr int kStStages = 4;
constexpr uint32_t kStStageBytes = 32768;
constexpr int kStConsumers = 4;
constexpr int kStThreads = (kStConsumers + 1) * 32;
constexpr int kStMaxContrib = 8;
constexpr size_t kStSmem = kStStages * kStStageBytes + 1024 + 256;
constexpr int kStPlane = kStRows * 16;  // one [64 rows][16 x rows] fp32 partial
constexpr size_t kStCtaSlotBytes = 2 /*first, last block*/ * 2 /*gate, up*/ * kStPlane * 4;

struct StreamArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  __nv_bfloat16* y[kMaxSeg];
  int64_t ldy[kMaxSeg];
  const __nv_bfloat16* bias[kMaxSeg];
  int row0[kMaxSeg + 1];  // segment starts in the concatenated row space (multiples of 64)
  int nseg;
  int m, k;
  int nkc;    // k chunks per row block
  int units;  // row blocks * nkc
  int ctas;
  float* slots;   // [ctas][first, last][gate, up][64][16]
  unsigned* cnt;  // [row blocks], zero between calls (after the slots)
  uint32_t* err;
  int weights_ready;  // the weights may be read before the previous kernel completes
  // Optional residual added in the epilogue of a single plain GEMV: y = W x + res.
  const __nv_bfloat16* res;
  int64_t ldres;
  long long wait_limit;  // SM cycles a bounded wait may take before the CTA unwinds
  int stall;             // test hook: CTA 0 skips the loads of its first unit
  int no_fast;           // test hook: every split row block takes the general merge
};

__device__ __forceinline__ int st_unit_begin(int c, const StreamArgs& a) {
  return static_cast<int>((static_cast<long long>(c) * a.units) / a.ctas);
}
// CTA whose range holds unit u.
__device__ __forceinline__ int st_cta_of(int u, const StreamArgs& a) {
  return static_cast<int>(((static_cast<long long>(u) + 1) * a.ctas + a.units - 1) / a.units) - 1;
}
__device__ __forceinline__ int st_segment(int row, const StreamArgs& a) {
  int si = 0;
  while (si + 1 < a.nseg && row >= a.row0[si + 1]) ++si;
  return si;
}

template <int MC, bool kGated>
__global__ void __launch_bounds__(kStThreads, 1)
    gemv_stream_kernel(const __grid_constant__ CUtensorMap m0,
                       const __grid_constant__ CUtensorMap m1,
                       const __grid_constant__ CUtensorMap m2, StreamArgs a) {
  constexpr int kKC = kGated ? 128 : 256;  // k columns per unit
  constexpr int kSlabs = kKC / 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStStages * kStStageBytes);
  // flags[0]: abort, flags[1]: "this CTA finishes the current row block", flags[2]: "the
  // other contributor of the last row block has posted its partial"
  volatile int* flags = reinterpret_cast<volatile int*>(bars + 2 * kStStages);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStStages);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int u0 = st_unit_begin(c, a), u1 = st_unit_begin(c + 1, a);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kStConsumers);
    }
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&m0);
    if (kGated || a.nseg > 1) prefetch_map(&m1);
    if (a.nseg > 2) prefetch_map(&m2);
  }
  __syncthreads();
  // The next kernel in the stream may begin its own prologue now.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == kStConsumers) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      if (!a.weights_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool issued = false, ok = true;
      for (int u = u0; u < u1; ++u) {
        const int rb = u / a.nkc, kc = u - rb * a.nkc;
        const int si = st_segment(rb * kStRows, a);
        const CUtensorMap* map = si == 0 ? &m0 : (si == 1 ? &m1 : &m2);
        const int rin = rb * kStRows - a.row0[si];
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, a.err, flags, a.wait_limit)) {
          ok = false;
          break;
        }
        const uint32_t fb = full0 + 8 * stage;
        const uint32_t dst = sbase + stage * kStStageBytes;
        mbar_expect_tx(fb, kStStageBytes);  // out-of-range rows / columns arrive as zeros
        if (a.stall && c == 0 && u == u0) {
          // Test hook (umic_debug_stall): the bytes are announced but never loaded, so the
          // consumers' wait on this stage runs out and the CTA unwinds.
        } else if constexpr (kGated) {
          tma_load_2d(dst, &m0, fb, kc * kKC, rin);
          tma_load_2d(dst + 8192, &m0, fb, kc * kKC + 64, rin);
          tma_load_2d(dst + 16384, &m1, fb, kc * kKC, rin);
          tma_load_2d(dst + 24576, &m1, fb, kc * kKC + 64, rin);
        } else {
#pragma unroll
          for (int b = 0; b < 4; ++b) tma_load_2d(dst + b * 8192, map, fb, kc * kKC + b * 64, rin);
        }
        issued = true;
        if (++stage == kStStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) {
        // Every stage released by the consumers before the CTA may exit.
        for (int s = 0; s < kStStages; ++s) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, a.err, flags, a.wait_limit)) break;
          if (++stage == kStStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      } else if (issued) {
        // Aborting: give copies in flight time to land before shared memory goes away.
        const long long t0 = clock64();
        while (clock64() - t0 < 4000000LL) {
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  const int r0 = warp * 16 + g, r1 = r0 + 8;  // rows inside the 64-row block
  float acc[MC][4], acc2[kGated ? MC : 1][4];
  auto zero_acc = [&]() {
#pragma unroll
    for (int i = 0; i < MC; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[i][j] = 0.f;
        if constexpr (kGated) acc2[i][j] = 0.f;
      }
  };
  zero_acc();
  const uint4 zero = make_uint4(0, 0, 0, 0);
  // x, y and the workspace may still belong to the previous kernel in the stream.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // The last row block of this CTA's range, when it has exactly one other contributor
  // and that one has already posted its partial: its partial is fetched while this CTA
  // streams its own last units (oth), and the block is summed and written without the
  // count round trip. fast == false keeps the general path below.
  constexpr int kVals = MC * 4 * (kGated ? 2 : 1);
  const int rb_last = u1 > u0 ? (u1 - 1) / a.nkc : -1;
  bool fast = false;
  bool fast_first = false;  // this CTA is the block's first contributor
  float oth[kVals];
  // slot 0 holds a CTA's first row block, slot 1 its last one
  auto slot_for = [&](int cta, int rb) {
    const int side = (rb == st_unit_begin(cta, a) / a.nkc) ? 0 : 1;
    return a.slots + (static_cast<size_t>(cta) * 2 + side) * 2 * kStPlane;
  };
  auto try_fast = [&](int rb) {
    const int first = st_cta_of(rb * a.nkc, a), last = st_cta_of((rb + 1) * a.nkc - 1, a);
    if (last - first != 1) return;
    if (warp == 0 && lane == 0) {
      // acquire: pairs with the other contributor's release of the count
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.cnt + rb) : "memory");
      flags[2] = v == 1u;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kStConsumers * 32) : "memory");
    if (!flags[2]) return;
    fast = true;
    fast_first = first == c;
    const float* src = slot_for(fast_first ? last : first, rb);
#pragma unroll
    for (int mc = 0; mc < MC; ++mc)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int rr = j < 2 ? r0 : r1, mcol = mc * 8 + 2 * t + (j & 1);
        oth[mc * 4 + j] = __ldcg(src + rr * 16 + mcol);
        if constexpr (kGated) oth[MC * 4 + mc * 4 + j] = __ldcg(src + kStPlane + rr * 16 + mcol);
      }
  };

  // Writes row block rb: directly when this CTA holds all of it, else via the slots.
  auto flush = [&](int rb) {
    const int first = st_cta_of(rb * a.nkc, a), last = st_cta_of((rb + 1) * a.nkc - 1, a);
    const int contrib = last - first + 1;
    const int si = st_segment(rb * kStRows, a);
    const int rows_in_seg = a.row0[si + 1] - a.row0[si];
    const int rin = rb * kStRows - a.row0[si];
    auto emit = [&](int rr, int mcol, float v, float v2) {
      const int nrow = rin + rr;
      if (nrow >= rows_in_seg || mcol >= a.m) return;
      float o;
      if constexpr (kGated) {
        o = v / (1.f + __expf(-v)) * v2;
      } else {
        o = v;
        if (a.bias[si]) o += bf(a.bias[si][nrow]);
        if (a.res) o += bf(a.res[mcol * a.ldres + nrow]);
      }
      a.y[si][mcol * a.ldy[si] + nrow] = __float2bfloat16_rn(o);
    };
    if (contrib == 1) {
#pragma unroll
      for (int mc = 0; mc < MC; ++mc)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          emit(j < 2 ? r0 : r1, mc * 8 + 2 * t + (j & 1), acc[mc][j], kGated ? acc2[mc][j] : 0.f);
      return;
    }
    if (fast && rb == rb_last) {
      // the same sums, in the same CTA order, as the general path below
#pragma unroll
      for (int mc = 0; mc < MC; ++mc)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float o1 = oth[mc * 4 + j], o2 = kGated ? oth[MC * 4 + mc * 4 + j] : 0.f;
          const float m1 = acc[mc][j], m2 = kGated ? acc2[mc][j] : 0.f;
          float v = 0.f, v2 = 0.f;
          v += fast_first ? m1 : o1;
          v += fast_first ? o1 : m1;
          if constexpr (kGated) {
            v2 += fast_first ? m2 : o2;
            v2 += fast_first ? o2 : m2;
          }
          emit(j < 2 ? r0 : r1, mc * 8 + 2 * t + (j & 1), v, v2);
        }
      if (warp == 0 && lane == 0) a.cnt[rb] = 0;  // both contributors are done with it
      return;
    }
    auto slot_of = [&](int cta) { return slot_for(cta, rb); };
    float* mine = slot_of(c);
#pragma unroll
    for (int mc = 0; mc < MC; ++mc)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int rr = j < 2 ? r0 : r1, mcol = mc * 8 + 2 * t + (j & 1);
        __stcg(mine + rr * 16 + mcol, acc[mc][j]);
        if constexpr (kGated) __stcg(mine + kStPlane + rr * 16 + mcol, acc2[mc][j]);
      }
    asm volatile("bar.sync 1, %0;" ::"n"(kStConsumers * 32) : "memory");
    if (warp == 0 && lane == 0) {
      // release: the partial stored above (ordered by the barrier) is visible with the
      // count; acquire: the last arrival sees every other contributor's partial
      unsigned prev;
      asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                   : "=r"(prev)
                   : "l"(a.cnt + rb)
                   : "memory");
      flags[1] = prev == static_cast<unsigned>(contrib - 1);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kStConsumers * 32) : "memory");
    if (!flags[1]) return;
    // All partial loads in flight at once, then sums in CTA order.
    float part[kStMaxContrib][kVals];
#pragma unroll
    for (int q = 0; q < kStMaxContrib; ++q) {
      if (q < contrib) {
        const float* src = slot_of(first + q);
#pragma unroll
        for (int mc = 0; mc < MC; ++mc)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int rr = j < 2 ? r0 : r1, mcol = mc * 8 + 2 * t + (j & 1);
            part[q][mc * 4 + j] = __ldcg(src + rr * 16 + mcol);
            if constexpr (kGated) part[q][MC * 4 + mc * 4 + j] = __ldcg(src + kStPlane + rr * 16 + mcol);
          }
      }
    }
#pragma unroll
    for (int mc = 0; mc < MC; ++mc)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v = 0.f, v2 = 0.f;
#pragma unroll
        for (int q = 0; q < kStMaxContrib; ++q) {
          if (q < contrib) {
            v += part[q][mc * 4 + j];
            if constexpr (kGated) v2 += part[q][MC * 4 + mc * 4 + j];
          }
        }
        emit(j < 2 ? r0 : r1, mc * 8 + 2 * t + (j & 1), v, v2);
      }
    asm volatile("bar.sync 1, %0;" ::"n"(kStConsumers * 32) : "memory");
    if (warp == 0 && lane == 0) {
      a.cnt[rb] = 0;  // ready for the next call
      flags[1] = 0;
    }
  };

  int stage = 0;
  uint32_t phase = 0;
  int cur = -1;
  for (int u = u0; u < u1; ++u) {
    const int rb = u / a.nkc, kc = u - rb * a.nkc;
    if (rb != cur) {
      if (cur >= 0) {
        flush(cur);
        zero_acc();
      }
      cur = rb;
      if (rb == rb_last && !a.no_fast) try_fast(rb);
    }
    // this chunk's activations, requested before the weights land
    uint4 xv[kSlabs][MC];
#pragma unroll
    for (int s = 0; s < kSlabs; ++s) {
      const int kk = kc * kKC + s * 32 + t * 8;
#pragma unroll
      for (int mc = 0; mc < MC; ++mc) {
        const int xr = mc * 8 + g;
        const bool live = kk < a.k && xr < a.m;
        xv[s][mc] = live ? ld_cached(a.x + xr * a.ldx + kk) : zero;
      }
    }
    // Every consumer warp passes or fails the same waits, so none is left alone at a
    // named barrier when another gives up.
    if (!mbar_wait(full0 + 8 * stage, phase, a.err, flags, a.wait_limit)) return;
    const uint32_t st = sbase + stage * kStStageBytes;
#pragma unroll
    for (int s = 0; s < kSlabs; ++s) {
      const uint32_t box = st + (s >> 1) * 8192;
      const int chunk = (s & 1) * 4 + t;
      const uint4 wl = lds128(st_swz(box, r0, chunk));
      const uint4 wh = lds128(st_swz(box, r1, chunk));
#pragma unroll
      for (int mc = 0; mc < MC; ++mc) slab_mma(acc[mc], wl, wh, xv[s][mc]);
      if constexpr (kGated) {
        const uint4 ul = lds128(st_swz(box + 16384, r0, chunk));
        const uint4 uh = lds128(st_swz(box + 16384, r1, chunk));
#pragma unroll
        for (int mc = 0; mc < MC; ++mc) slab_mma(acc2[mc], ul, uh, xv[s][mc]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * stage);
    if (++stage == kStStages) {
      stage = 0;
      phase ^= 1;
    }
  }
  if (cur >= 0) flush(cur);
}

inline size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Workspace of the streaming engine: one pair of partial slots per CTA (one CTA
// per SM), then the row-block counters. The counters sit at the same offset for
// every call on a device, so a call with more row blocks than any before it finds
// zeros there (slots are never written over counters).
size_t stream_counter_offset() {
  return align256(static_cast<size_t>(sm_count()) * kStCtaSlotBytes);
}
size_t stream_workspace_bytes(int64_t rows) {
  const int64_t blocks = (rows + kStRows - 1) / kStRows;
  return stream_counter_offset() + align256(static_cast<size_t>(blocks) * 4);
}

// The streaming engine covers m <= 16 and segment starts on 64-row boundaries.
bool stream_eligible(const GemvArgs& a) {
  if (a.m > 16) return false;
  for (int i = 1; i < a.nseg; ++i)
    if (a.seg[i].row0 % kStRows) return false;
  return true;
}

template <int MC, bool kGated>
int stream_launch(const char* name, const GemvArgs& a, void* ws, size_t ws_bytes,
                  uint32_t flags, cudaStream_t st, bool pdl = true,
                  const StreamArgs* extra = nullptr) {
  static std::once_flag attr_once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once[dev >= 0 && dev < 64 ? dev : 0], [&] {
    attr_err = cudaFuncSetAttribute(gemv_stream_kernel<MC, kGated>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kStSmem));
  });
  if (attr_err != cudaSuccess)
    return fail(UMIC_ERR_LAUNCH, "%s: smem attribute: %s", name, cudaGetErrorString(attr_err));
  CUtensorMap maps[kMaxSeg];
  for (int i = 0; i < kMaxSeg; ++i) {
    const Seg& sg = a.seg[i < a.nseg ? i : 0];
    const void* base = (kGated && i == 1) ? static_cast<const void*>(a.w2) : sg.w;
    if (!make_map(&maps[i], base, sg.rows, a.k, sg.ldw, kStRows))
      return fail(UMIC_ERR_DEVICE, "%s: cuTensorMapEncodeTiled unavailable or rejected", name);
  }
  StreamArgs s{};
  s.x = a.x;
  s.ldx = a.ldx;
  for (int i = 0; i < a.nseg; ++i) {
    s.y[i] = a.seg[i].y;
    s.ldy[i] = a.seg[i].ldy;
    s.bias[i] = a.seg[i].bias;
    s.row0[i] = a.seg[i].row0;
  }
  s.row0[a.nseg] = a.n;
  s.nseg = a.nseg;
  s.m = a.m;
  s.k = a.k;
  constexpr int kKC = kGated ? 128 : 256;
  s.nkc = (a.k + kKC - 1) / kKC;
  const int64_t blocks = (static_cast<int64_t>(a.n) + kStRows - 1) / kStRows;
  const int64_t units = blocks * s.nkc;
  if (units > 0x7fffffffLL / 256)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: matrix too large for the streaming engine", name);
  s.units = static_cast<int>(units);
  // At least ceil(nkc / 7) units per CTA keeps a row block within 8 contributors.
  const int per = (s.nkc + kStMaxContrib - 2) / (kStMaxContrib - 1);
  const int64_t by_units = units / per;
  s.ctas = static_cast<int>(by_units < sm_count() ? (by_units > 0 ? by_units : 1) : sm_count());
  const size_t need = stream_workspace_bytes(a.n);
  if (ws_bytes < need)
    return fail(UMIC_ERR_INVALID_ARG, "%s: workspace of %zu bytes, %zu needed", name, ws_bytes,
                need);
  if (reinterpret_cast<uintptr_t>(ws) & 255u)
    return fail(UMIC_ERR_ALIGNMENT, "%s: workspace must be 256-byte aligned", name);
  s.slots = static_cast<float*>(ws);
  s.cnt = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + stream_counter_offset());
  s.err = device_error_word();
  s.weights_ready = (flags & UMIC_GEMV_WEIGHTS_READY) ? 1 : 0;
  s.wait_limit = kWaitLimitCycles;
  s.stall = 0;
  {
    long long limit = 0;
    if (take_stall(kStallGemv, &limit)) {
      s.stall = 1;
      s.wait_limit = limit;
    }
    s.no_fast = take_stall(kGemvGeneralMerge, &limit) ? 1 : 0;
  }
  if (extra) {  // residual epilogue
    s.res = extra->res;
    s.ldres = extra->ldres;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(s.ctas, 1, 1);
  cfg.blockDim = dim3(kStThreads, 1, 1);
  cfg.dynamicSmemBytes = kStSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_stream_kernel<MC, kGated>, maps[0], maps[1],
                                     maps[2], s);
  if (e != cudaSuccess) return fail(UMIC_ERR_LAUNCH, "%s: %s", name, cudaGetErrorString(e));
  return launch_status(name);
}

// ------------------------------------------------------- allocation-free entry
//
// umic_gemv_noalloc runs the streaming engine on a scratch area that is part of
// the library image: a file-scope __device__ array, created with the module on
// each device, so the call itself allocates nothing. It serves hosts that may not
// allocate device memory at call time (a real-time control loop that reserved its
// memory at start-up, an FFI runtime that owns its device pool). Its size bounds
// the calls it takes (rows per call and SMs per device). One array per device
// serves every such call on that device, from any stream or thread: calls that
// overlap on the GPU race. Host code may not pass g_gemv_scratch itself to a
// kernel (its host-side name is a stand-in, not a device address); the address
// comes from cudaGetSymbolAddress, on the first call on each device.
constexpr int64_t kStaticMaxRows = int64_t{1} << 20;
constexpr int kStaticMaxSms = 256;
constexpr size_t kStaticScratchBytes =
    kStaticMaxSms * kStCtaSlotBytes + static_cast<size_t>(kStaticMaxRows / kStRows) * 4;
static __device__ __align__(256) unsigned char g_gemv_scratch[kStaticScratchBytes];

// Device address of g_gemv_scratch on the current device, resolved once per device
// (with that device current).
int static_scratch(const char* name, void** out) {
  static std::once_flag once[64];
  static void* addr[64];
  static cudaError_t status[64];
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(UMIC_ERR_DEVICE, "%s: cudaGetDevice: %s", name,
                                    cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(UMIC_ERR_UNSUPPORTED, "%s: device %d", name, dev);
  std::call_once(once[dev], [dev] {
    status[dev] = cudaGetSymbolAddress(&addr[dev], g_gemv_scratch);
    if (status[dev] != cudaSuccess) cudaGetLastError();
  });
  if (status[dev] != cudaSuccess)
    return fail(UMIC_ERR_DEVICE, "%s: cudaGetSymbolAddress of the static scratch: %s", name,
                cudaGetErrorString(status[dev]));
  *out = addr[dev];
  return UMIC_OK;
}

// Engine choice: streaming with a workspace, cluster split-K without one (or for
// shapes the streaming engine does not cover).
template <bool kGated>
int run(const char* name, const GemvArgs& a, void* ws, size_t ws_bytes, uint32_t flags,
        cudaStream_t st) {
  if (flags & ~static_cast<uint32_t>(UMIC_GEMV_WEIGHTS_READY))
    return fail(UMIC_ERR_INVALID_ARG, "%s: unknown flags 0x%x", name, flags);
  if (ws && stream_eligible(a))
    return a.m <= 8 ? stream_launch<1, kGated>(name, a, ws, ws_bytes, flags, st)
                    : stream_launch<2, kGated>(name, a, ws, ws_bytes, flags, st);
  return dispatch<kGated>(a, st);
}

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" {

int umic_gemv(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias, void* y,
              int64_t ldy, int64_t m, int64_t n, int64_t k, void* workspace,
              size_t workspace_bytes, uint32_t flags, void* stream) {
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
  return run<false>("umic_gemv", a, workspace, workspace_bytes, flags, as_stream(stream));
}

int umic_gemv_multi(const void* x, int64_t ldx, int32_t count, const void* const* w,
                    const int64_t* ldw, const int64_t* n, const void* const* bias,
                    void* const* y, const int64_t* ldy, int64_t m, int64_t k, void* workspace,
                    size_t workspace_bytes, uint32_t flags, void* stream) {
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
  return run<false>("umic_gemv_multi", a, workspace, workspace_bytes, flags,
                    as_stream(stream));
}

int umic_gemv_gate_silu_mul(const void* x, int64_t ldx, const void* wg, const void* wu,
                            int64_t ldw, void* h, int64_t ldh, int64_t m, int64_t n, int64_t k,
                            void* workspace, size_t workspace_bytes, uint32_t flags,
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
  return run<true>("umic_gemv_gate_silu_mul", a, workspace, workspace_bytes, flags,
                   as_stream(stream));
}

int umic_gemv_noalloc(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
                      void* y, int64_t ldy, int64_t m, int64_t n, int64_t k, void* stream) {
  static const char* kName = "umic_gemv_noalloc";
  clear_error();
  if (int rc = check(kName, x, ldx, w, w, ldw, y, ldy, m, n, k)) return rc;
  if (m == 0 || n == 0) return UMIC_OK;
  if (m > 16)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: m=%lld rows of x; the streaming engine takes 1..16",
                kName, (long long)m);
  if (n > kStaticMaxRows)
    return fail(UMIC_ERR_UNSUPPORTED,
                "%s: n=%lld weight rows exceed the static scratch maximum of %lld rows", kName,
                (long long)n, (long long)kStaticMaxRows);
  if (sm_count() > kStaticMaxSms)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: %d SMs exceed the static scratch maximum of %d",
                kName, sm_count(), kStaticMaxSms);
  void* scratch = nullptr;
  if (int rc = static_scratch(kName, &scratch)) return rc;
  cudaStream_t st = as_stream(stream);
  // The row-block counters must start at zero: clear this call's range on the stream
  // (a kernel that ran out of its wait limit may have left some set).
  const size_t counters = align256(static_cast<size_t>((n + kStRows - 1) / kStRows) * 4);
  cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + stream_counter_offset(), 0,
                                  counters, st);
  if (e != cudaSuccess)
    return fail(UMIC_ERR_LAUNCH, "%s: clearing the counters: %s", kName, cudaGetErrorString(e));
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
  // Plain stream order (no programmatic dependent launch): the memset above must
  // complete before any CTA reads a counter.
  return a.m <= 8 ? stream_launch<1, false>(kName, a, scratch, kStaticScratchBytes, 0, st, false)
                  : stream_launch<2, false>(kName, a, scratch, kStaticScratchBytes, 0, st, false);
}

int umic_gemv_residual(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
                       const void* res, int64_t ldres, void* y, int64_t ldy, int64_t m, int64_t n,
                       int64_t k, void* workspace, size_t workspace_bytes, uint32_t flags,
                       void* stream) {
  static const char* kName = "umic_gemv_residual";
  clear_error();
  if (!res) return fail(UMIC_ERR_INVALID_ARG, "%s: res is null", kName);
  if (int rc = check(kName, x, ldx, w, w, ldw, y, ldy, m, n, k)) return rc;
  if (m == 0 || n == 0) return UMIC_OK;
  if (m > 16)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: m=%lld rows of x; 1..16 supported", kName,
                (long long)m);
  if (!aligned16(res) || ldres < n)
    return fail(UMIC_ERR_ALIGNMENT, "%s: res must be 16-byte aligned with ldres >= n", kName);
  if (!workspace)
    return fail(UMIC_ERR_INVALID_ARG, "%s: needs a workspace (streaming engine)", kName);
  if (flags & ~static_cast<uint32_t>(UMIC_GEMV_WEIGHTS_READY))
    return fail(UMIC_ERR_INVALID_ARG, "%s: unknown flags 0x%x", kName, flags);
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
  if (!stream_eligible(a))
    return fail(UMIC_ERR_UNSUPPORTED, "%s: shape outside the streaming engine", kName);
  StreamArgs extra{};
  extra.res = static_cast<const __nv_bfloat16*>(res);
  extra.ldres = ldres;
  cudaStream_t st = as_stream(stream);
  return a.m <= 8 ? stream_launch<1, false>(kName, a, workspace, workspace_bytes, flags, st, true,
                                            &extra)
                  : stream_launch<2, false>(kName, a, workspace, workspace_bytes, flags, st, true,
                                            &extra);
}

size_t umic_gemv_workspace_bytes(int64_t rows) {
  clear_error();
  if (rows < 0) return 0;
  return stream_workspace_bytes(rows);
}

}  // extern "C"
