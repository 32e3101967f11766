// Tensor-core GEMM for sm_100a: tcgen05.mma with TMEM accumulators, fed by TMA.
//
//   y[m, n] = epi(sum_k x[m, k] * w[n, k] + bias[n]) + residual[m, n]    (linear)
//   h[m, n] = silu(x . wg[n]) * (x . wu[n])                              (gate/up)
//
// Both operands are K-major (activations [m, k] row-major, nn.Linear weights
// [n, k] row-major), so no transpose or copy of the weights is ever made.
//
// Persistent kernel, one CTA per SM, 6 warps with fixed roles. For m > 128 the CTAs
// run as pairs (cta_group::2): a pair computes a 256 x 256 tile with one M = 256,
// N = 256, K = 16 MMA per 16-wide k-step, each CTA staging its 128 rows of A and half
// of B; one-block shapes (m <= 128) use single CTAs with M = 128 tiles.
//   warp 0     TMA producer: fills the shared-memory ring (6 stages of 32 KB per
//              CTA for pairs: A 128x64 + B 128x64; 4 stages of 48 KB for single
//              CTAs: A 128x64 + B 256x64), bf16, 128-byte swizzled;
//   warp 1     allocates 512 TMEM columns; in the pair's leader CTA one lane issues
//              tcgen05.mma (4 per 64-wide k-block) and commits each stage back to
//              both CTAs' producers through their mbarriers;
//   warps 2-5  epilogue: tcgen05.ld of the fp32 accumulator (each warp reads
//              its 32-lane TMEM quarter), bias / activation / residual in
//              registers, then the bf16 32 x 32 chunk is staged in shared
//              memory (64-byte swizzle, double-buffered per warp) and written
//              with one TMA store, so output leaves in full lines instead of
//              32 scattered 16-byte pieces per instruction.
// The accumulator is double-buffered in TMEM (2 x 256 columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// Gate/up: the B stage holds 128 rows of w_gate followed by 128 rows of w_up
// (two TMA loads into adjacent 16 KB halves). One N=256 MMA then produces the
// gate accumulator in TMEM columns 0-127 and the up accumulator in 128-255;
// the epilogue combines them as silu(g) * u, so neither product reaches HBM
// (the reference's dual accumulators, fused_ffn.py:68-87).
//
// Tiles are walked in groups of kGroupM row-blocks (row-block fastest) so a
// wave of CTAs shares both its activation rows and its weight columns in L2
// (the reference's GROUP swizzle, linear.py:43-55).
//
// Split-K (umic_gemm_ws, linear only): when the output tiles would keep at most
// half of the CTA pairs busy, each tile's k-blocks are cut into up to kMaxSplits
// ranges, one work unit per CTA (pair), so every unit is resident at once. A unit
// owns whole 32-column chunks of its tile; it posts its fp32 partials of the
// other units' chunks to the workspace, counts itself in, waits (bounded) for
// the others, bulk-copies their partials of its own chunks into its idle stage
// ring and sums them in range order, so the result does not depend on timing.
//
// Launch order: the kernel is launched with programmatic stream serialization.
// It sets up its barriers and TMEM, lets the stream's next kernel begin its own
// set-up, then waits for the previous kernel (griddepcontrol.wait) before its
// first load.
//
// Every mbarrier wait is bounded (about 5 s of SM clock); a wait that runs
// out sets UMIC_DEVERR_WAIT_TIMEOUT, the CTA drains its outstanding work,
// frees its TMEM and exits instead of hanging.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "tma.cuh"

namespace umic {
namespace {

constexpr int kBM = 128;   // accumulator rows per CTA (TMEM lanes)
constexpr int kBN = 256;   // MMA N (output tile width for linear; 2 x 128 for gate/up)
constexpr int kBK = 64;    // one 128-byte swizzle atom of bf16
constexpr int kThreads = 192;
constexpr int kGroupM = 16;
constexpr int kMaxSplits = 8;  // k ranges per tile at most (split-K): one 32-column
                               // chunk of the tile at least per range
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB

// Per-variant geometry. kPair = 2 runs one MMA over a CTA pair (cta_group::2):
// the pair computes a 256 x 256 tile, each CTA holding its 128 rows of A and
// half (128 rows) of B, so a CTA stages 32 KB per k-block instead of 48 KB.
template <int kPair>
struct Geo {
  static constexpr uint32_t kBBytes = kBN * kBK * 2 / kPair;  // B rows held by one CTA
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kPair == 2 ? 6 : 4;
  static constexpr uint32_t kBarBytes = 1024;                       // barriers + flags
  static constexpr uint32_t kStageOut = kStages * kStageBytes + kBarBytes;  // output staging
  static constexpr uint32_t kOutBytes = 4 * 2 * 32 * 64;              // 4 warps x 2 x [32 x 32] bf16
  static constexpr size_t kSmem = kStageOut + kOutBytes + 1024 /*align*/;
  static constexpr int kTileM = kBM * kPair;
  // D fp32, A/B bf16, both K-major, N = 256, M = 128 x kPair
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((kBN >> 3) << 17) |
                                     (((kBM * kPair) >> 4) << 24);
};

struct TcParams {
  __nv_bfloat16* y;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  int64_t ldy, ldr;
  uint32_t* err;
  int m, n, k;
  int tiles_m, tiles_n;  // output tiles
  int kblocks;
  int epilogue;
  long long wait_limit;  // SM cycles a bounded wait may take before the CTA unwinds
  int stall;             // test hook: CTA 0 skips the loads of its first stage
  // Split-K (linear only): each tile's k-blocks are cut into `splits` contiguous ranges,
  // one work unit each; a unit writes its fp32 partial of the column chunks other units
  // own to `part`, waits until the tile half's other units have written theirs (counted
  // in `cnt`), then sums its own chunks over all partials in range order and runs the
  // epilogue on them.
  int splits;
  float* part;    // [tiles][2 halves][splits][4 warps][8 chunks][8][32 lanes] float4
  unsigned* cnt;  // [tiles][2 halves][arrived, done], zero between calls
};

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row
// core-matrix groups 1024 bytes apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;           // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;   // SBO
  d |= static_cast<uint64_t>(1) << 46;           // version
  d |= static_cast<uint64_t>(2) << 61;           // SWIZZLE_128B
  return d;
}

template <int kPair>
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
  if constexpr (kPair == 2) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(Geo<2>::kIdesc), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(Geo<1>::kIdesc), "r"(accumulate));
  }
}

// Arrive on `bar` (a shared::cluster address, possibly in the peer CTA) once every
// tcgen05 operation issued so far by this thread has completed.
template <int kPair>
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  if constexpr (kPair == 2) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
  } else {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
  }
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(local), "r"(rank));
  return out;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Remote (or local) arrive on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
               : "memory");
}

// TMA load of a CTA-pair operand: lands in this CTA's shared memory and counts
// its bytes on the leader CTA's barrier `bar` (a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ float4 lds_f4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t a, const uint4& v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w) : "memory");
}

// 32 lanes x 32 consecutive fp32 columns; thread i receives lane (base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tile_coords(int t, const TcParams& p, int& mb, int& nb) {
  const int per_group = kGroupM * p.tiles_n;
  const int g = t / per_group;
  const int first = g * kGroupM;
  const int gm = min(p.tiles_m - first, kGroupM);
  const int r = t - g * per_group;
  mb = first + r % gm;
  nb = r / gm;
}

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
}
// tanh on the SFU (PTX tanh.approx.f32, relative error about 2^-11, far below the bf16
// rounding of the output): the ViT fc1 epilogue evaluates one per element, and the
// multi-instruction library tanhf left that epilogue longer than the tile's MMAs at K = 1280.
__device__ __forceinline__ float tanh_sfu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.f + tanh_sfu(u));
}
__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// ------------------------------------------------------------------ kernel

template <bool kDual, int kPair>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_b2,
                   const __grid_constant__ CUtensorMap map_y, TcParams p) {
  using G = Geo<kPair>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kStages * G::kStageBytes);
  // bars: full[kStages], empty[kStages], acc_full[2], acc_empty[2], drain
  // bars[2 * kStages + 8 ...+ 11]: split-K partial fetches, one per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * G::kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;  // split-K: this CTA sums the tile half

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = kPair == 2 ? cluster_rank() : 0;  // position in the CTA pair
  const bool leader = rank == 0;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + G::kStages);
  const uint32_t accf0 = smem_u32(bars + 2 * G::kStages), acce0 = accf0 + 16;
  const uint32_t drain = accf0 + 32;
  const uint32_t red0 = smem_u32(bars + 2 * G::kStages + 8);
  const uint32_t sbase = smem_u32(smem);
  const int tiles = p.tiles_m * p.tiles_n;
  const int work = tiles * p.splits;  // work units: (tile, k range)
  const int unit = kPair == 2 ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
  const int units = kPair == 2 ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < G::kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accf0, 1);
    mbar_init(accf0 + 8, 1);
    mbar_init(acce0, 128 * kPair);  // every epilogue thread of the pair
    mbar_init(acce0 + 8, 128 * kPair);
    mbar_init(drain, 1);
    for (int q = 0; q < 4; ++q) mbar_init(red0 + 8 * q, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    prefetch_map(&map_a);
    prefetch_map(&map_b);
    if (kDual) prefetch_map(&map_b2);
  }
  if (warp == 1) {
    if constexpr (kPair == 2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  if constexpr (kPair == 2) cluster_sync_all();  // peer barriers initialised before any use
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The set-up above overlaps the previous kernel's tail (the launch allows it); the
  // operands, the output and the split-K workspace are touched only after it completed.
  allow_dependent_launch();
  wait_prerequisite();
  // The leader's barriers as seen from either CTA of the pair.
  const uint32_t lead_full0 = kPair == 2 ? cluster_addr(full0, 0) : full0;
  const uint32_t lead_acce0 = kPair == 2 ? cluster_addr(acce0, 0) : acce0;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      for (int w = unit; w < work && ok; w += units) {
        const int t = w / p.splits, sp = w - t * p.splits;
        const int kb0 = sp * p.kblocks / p.splits, kb1 = (sp + 1) * p.kblocks / p.splits;
        int mb, nb;
        tile_coords(t, p, mb, nb);
        const int row_a = mb * G::kTileM + static_cast<int>(rank) * kBM;
        int row_b;
        const CUtensorMap* bmap = &map_b;
        if (kDual) {
          row_b = nb * (kBN / 2);
          if (kPair == 2 && rank == 1) bmap = &map_b2;  // the pair's second half holds up
        } else {
          row_b = nb * kBN + static_cast<int>(rank) * (kBN / kPair);
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.err, abort_flag, p.wait_limit)) {
            ok = false;
            break;
          }
          const uint32_t sa = sbase + stage * G::kStageBytes;
          const uint32_t sb = sa + kABytes;
          // Test hook (umic_debug_stall): the stage's bytes are announced but CTA 0 never
          // loads them, so the MMA's wait on it runs out and the abort path unwinds.
          const bool skip = p.stall && blockIdx.x == 0 && !issued;
          if constexpr (kPair == 2) {
            const uint32_t fb = lead_full0 + 8 * stage;
            if (leader) mbar_expect_tx(full0 + 8 * stage, 2 * G::kStageBytes);
            if (!skip) {
              tma_load_2d_pair(sa, &map_a, fb, kb * kBK, row_a);
              tma_load_2d_pair(sb, bmap, fb, kb * kBK, row_b);
            }
          } else if (skip) {
            mbar_expect_tx(full0 + 8 * stage, G::kStageBytes);
          } else {
            const uint32_t fb = full0 + 8 * stage;
            mbar_expect_tx(fb, G::kStageBytes);
            tma_load_2d(sa, &map_a, fb, kb * kBK, row_a);
            if (kDual) {
              tma_load_2d(sb, &map_b, fb, kb * kBK, row_b);
              tma_load_2d(sb + G::kBBytes / 2, &map_b2, fb, kb * kBK, row_b);
            } else {
              tma_load_2d(sb, &map_b, fb, kb * kBK, row_b);
            }
          }
          issued = true;
          if (++stage == G::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (ok) {
        // Tail: wait until the MMA has released every stage this CTA filled, so no
        // commit from the (possibly peer) MMA thread is still in flight at exit.
        for (int s = 0; s < G::kStages; ++s) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.err, abort_flag, p.wait_limit)) break;
          if (++stage == G::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      } else if (issued) {
        // Aborting: give the copies already in flight time to land (they take
        // microseconds) before this CTA's shared memory is released.
        const long long t0 = clock64();
        while (clock64() - t0 < 4000000LL) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      const uint32_t peer = kPair == 2 ? 1u : 0u;
      for (int w = unit; w < work && ok; w += units, ++it) {
        const int t = w / p.splits, sp = w - t * p.splits;
        const int kb0 = sp * p.kblocks / p.splits, kb1 = (sp + 1) * p.kblocks / p.splits;
        (void)t;
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(acce0 + 8 * acc, acc_phase ^ 1, p.err, abort_flag, p.wait_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * kBN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase, p.err, abort_flag, p.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + stage * G::kStageBytes;
          const uint64_t ad = sdesc(sa), bd = sdesc(sa + kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // +32 bytes along K inside the swizzle atom = +2 in the >>4 field
            mma_bf16<kPair>(tmem_d, ad + 2 * kk, bd + 2 * kk, ((kb - kb0) | kk) ? 1u : 0u);
          }
          mma_commit<kPair>(empty0 + 8 * stage);  // frees this stage in both CTAs
          if (kPair == 2) mma_commit<kPair>(cluster_addr(empty0 + 8 * stage, peer));
          if (++stage == G::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) {
          mma_commit<kPair>(accf0 + 8 * acc);
          if (kPair == 2) mma_commit<kPair>(cluster_addr(accf0 + 8 * acc, peer));
        }
      }
      // Wait for every MMA issued by this thread before TMEM is released.
      mma_commit<kPair>(drain);
      mbar_wait(drain, 0, p.err, abort_flag, p.wait_limit);
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    // two [32 rows x 32 cols] bf16 staging buffers per epilogue warp for TMA stores
    const uint32_t stg0 = sbase + G::kStageOut + quarter * 4096;
    int chunk_idx = 0;
    int it = 0;
    uint32_t red_phase = 0;  // split-K partial fetch barrier parity
    constexpr int kOutCols = kDual ? kBN / 2 : kBN;
    const int erow = quarter * 32 + lane;  // this thread's accumulator row (TMEM lane)
    // Bias / activation / residual on one 32-column chunk of this thread's row, then the
    // warp's 32 x 32 chunk staged in shared memory (64-byte swizzle: 16-byte chunk j of
    // row r at j ^ ((r >> 1) & 3), conflict-free) and written with one TMA store.
    auto store_chunk = [&](float (&v)[32], int mb, int cbase) {
      const int row = mb * G::kTileM + static_cast<int>(rank) * kBM + erow;
      const bool live = row < p.m;  // rows past m hold zeros; the TMA store clips them
      if (!kDual) {
        if (p.bias) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            if (cbase + i < p.n) {
              float b[8];
              unpack8(ld_cached(p.bias + cbase + i), b);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i + j] += b[j];
            }
          }
        }
        if (p.epilogue == UMIC_EPI_GELU_ERF) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
        } else if (p.epilogue == UMIC_EPI_GELU_TANH) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
        }
        if (p.residual && live) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            if (cbase + i < p.n) {
              float r[8];
              unpack8(ld_stream(p.residual + static_cast<int64_t>(row) * p.ldr + cbase + i), r);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i + j] += r[j];
            }
          }
        }
      }
      const uint32_t buf = stg0 + (chunk_idx & 1) * 2048;
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float o[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) o[jj] = v[j * 8 + jj];
        st_shared_v4(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4), pack8(o));
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&map_y, buf, cbase,
                     mb * G::kTileM + static_cast<int>(rank) * kBM + quarter * 32);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
      ++chunk_idx;
    };
    for (int w = unit; w < work; w += units, ++it) {
      const int t = w / p.splits, sp = w - t * p.splits;
      int mb, nb;
      tile_coords(t, p, mb, nb);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(accf0 + 8 * acc, acc_phase, p.err, abort_flag, p.wait_limit)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN;
      const int col0 = nb * kOutCols;
      if (p.splits == 1) {
#pragma unroll 1
        for (int c = 0; c < kOutCols; c += 32) {
          __syncwarp();  // tcgen05.ld is warp-collective
          float v[32];
          tmem_ld32(tbase + c, v);
          if (kDual) {
            float u[32];
            tmem_ld32(tbase + kBN / 2 + c, u);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = silu(v[i]) * u[i];
          }
          if (c + 32 >= kOutCols) {
            // All TMEM reads of this tile are done: hand the buffer back to the MMA.
            tc_fence_before();
            if (kPair == 2) mbar_arrive_cluster(lead_acce0 + 8 * acc);
            else mbar_arrive(acce0 + 8 * acc);
          }
          store_chunk(v, mb, col0 + c);
        }
        continue;
      }
      if constexpr (!kDual) {
        // Split-K (every unit of the launch resident, at most one per CTA). The tile
        // half's 8 column chunks of 32 are dealt to its `splits` units as contiguous
        // ranges; a unit stores its partial of every chunk it does not own, counts itself
        // in, waits for the others, then fetches their partials of its own chunks with
        // bulk copies into its warp's quarter of the idle stage ring and sums them in unit
        // order (deterministic) with its own accumulator, still in TMEM.
        constexpr int kChunks = kOutCols / 32;
        const int s = p.splits;
        const int own_lo = sp * kChunks / s, own_hi = (sp + 1) * kChunks / s;
        // partial block (unit q, warp quarter, chunk): 32 rows x 32 fp32 as [8][32 lanes]
        // float4, so every warp store / load instruction covers 512 contiguous bytes
        float4* part_tile = reinterpret_cast<float4*>(p.part) +
                            (static_cast<size_t>(t) * 2 + rank) * s * 4 * kChunks * 256;
        auto block = [&](int q, int ci) {
          return part_tile + ((static_cast<size_t>(q) * 4 + quarter) * kChunks + ci) * 256;
        };
#pragma unroll 1
        for (int ci = 0; ci < kChunks; ++ci) {
          if (ci >= own_lo && ci < own_hi) continue;
          __syncwarp();
          float v[32];
          tmem_ld32(tbase + ci * 32, v);
          float4* dst = block(sp, ci) + lane;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(dst + j * 32, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
        }
        unsigned* cnt = p.cnt + static_cast<size_t>(t) * 4 + rank * 2;  // [arrived, done]
        __threadfence();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (quarter == 0 && lane == 0) {
          asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
          *last_flag = 1;
          const long long start = clock64();
          for (uint32_t i = 0;; ++i) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
            if (v >= static_cast<unsigned>(s)) break;
            if ((i & 63u) == 63u && clock64() - start > p.wait_limit) {
              *abort_flag = 1;
              if (p.err) atomicOr(p.err, UMIC_DEVERR_WAIT_TIMEOUT);
              *last_flag = 0;
              break;
            }
            __nanosleep(32);
          }
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (!*last_flag) break;  // a partner never arrived: unwind
        const uint32_t region = sbase + quarter * (G::kStages * G::kStageBytes / 4);
        const uint32_t rbar = red0 + 8 * quarter;
        if (lane == 0) {
          // the partials were written through the generic proxy by other SMs; order
          // their (acquired) visibility before this thread's async-proxy reads
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          asm volatile("fence.proxy.async.global;" ::: "memory");
          mbar_expect_tx(rbar, static_cast<uint32_t>((own_hi - own_lo) * (s - 1)) * 4096u);
          uint32_t slot = 0;
          for (int ci = own_lo; ci < own_hi; ++ci)
            for (int q = 0; q < s; ++q)
              if (q != sp) bulk_load(region + 4096u * slot++, block(q, ci), 4096u, rbar);
        }
        if (!mbar_wait(rbar, red_phase, p.err, abort_flag, p.wait_limit)) {
          // copies may still be in flight into this shared memory: let them land
          const long long t0 = clock64();
          while (clock64() - t0 < 4000000LL) {
          }
          break;
        }
        red_phase ^= 1;
        uint32_t slot = 0;
#pragma unroll 1
        for (int ci = own_lo; ci < own_hi; ++ci) {
          __syncwarp();
          float mine[32];
          tmem_ld32(tbase + ci * 32, mine);
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
#pragma unroll 1
          for (int q = 0; q < s; ++q) {
            if (q == sp) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += mine[i];
            } else {
              const uint32_t src = region + 4096u * slot++ + lane * 16;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 f = lds_f4(src + j * 512);
                v[4 * j] += f.x;
                v[4 * j + 1] += f.y;
                v[4 * j + 2] += f.z;
                v[4 * j + 3] += f.w;
              }
            }
          }
          store_chunk(v, mb, col0 + ci * 32);
        }
        tc_fence_before();
        if (kPair == 2) mbar_arrive_cluster(lead_acce0 + 8 * acc);
        else mbar_arrive(acce0 + 8 * acc);
        // the last unit to finish returns both counters to zero (every unit has passed
        // the wait above by then, so none reads them again)
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (quarter == 0 && lane == 0) {
          unsigned prev;
          asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                       : "=r"(prev)
                       : "l"(cnt + 1)
                       : "memory");
          if (prev == static_cast<unsigned>(s - 1)) {
            cnt[0] = 0;
            cnt[1] = 0;
          }
        }
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }

  tc_fence_before();
  // Neither CTA of a pair leaves (or frees TMEM) while the other may still touch
  // its barriers or shared memory.
  if constexpr (kPair == 2) cluster_sync_all();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair == 2) {
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(kTmemCols));
    } else {
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(kTmemCols));
    }
  }
}

// --------------------------------------------------------------------- host

template <bool kDual, int kPair>
int set_smem_attr() {
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  cudaError_t e = cudaSuccess;
  std::call_once(once[dev], [&] {
    e = cudaFuncSetAttribute(tc_gemm_kernel<kDual, kPair>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Geo<kPair>::kSmem));
  });
  if (e != cudaSuccess) return fail(UMIC_ERR_LAUNCH, "tc_gemm smem attribute: %s",
                                    cudaGetErrorString(e));
  return UMIC_OK;
}

int check_operand(const char* name, const char* what, const void* p, int64_t ld, int64_t k) {
  if (!p) return fail(UMIC_ERR_INVALID_ARG, "%s: %s is NULL", name, what);
  if (!aligned16(p)) return fail(UMIC_ERR_ALIGNMENT, "%s: %s not 16-byte aligned", name, what);
  if (ld % 8) return fail(UMIC_ERR_ALIGNMENT, "%s: ld of %s not a multiple of 8", name, what);
  if (ld < k) return fail(UMIC_ERR_INVALID_ARG, "%s: ld of %s < k", name, what);
  return UMIC_OK;
}

// Split-K plan of a linear launch: when the output tiles would fill at most half of the
// CTA pairs (or single CTAs), each tile's k-blocks are cut into `splits` ranges so the work
// units fill the GPU (at least 4 k-blocks per range, at most 8 ranges). 1 = no split.
// Counter area at the start of a split-K workspace: two words (arrived, done) per tile
// half for the at most 128 tiles a split launch has (tiles * 2 <= CTA pairs or CTAs).
constexpr size_t kSplitCounterBytes = 4096;

struct SplitPlan {
  int splits = 1;
  size_t part_bytes = 0, cnt_offset = 0, bytes = 0;  // counters at cnt_offset (0)
};

SplitPlan plan_split(int64_t m, int64_t n, int64_t k, int units_max) {
  SplitPlan sp;
  const bool pair = m > kBM;
  const int64_t tiles = ((m + (pair ? 2 * kBM : kBM) - 1) / (pair ? 2 * kBM : kBM)) *
                        ((n + kBN - 1) / kBN);
  const int64_t kblocks = (k + kBK - 1) / kBK;
  if (tiles <= 0 || tiles * 2 > units_max || kblocks < 8) return sp;
  int64_t s = units_max / tiles;
  if (s > kblocks / 4) s = kblocks / 4;
  if (s > kMaxSplits) s = kMaxSplits;
  if (s < 2) return sp;
  sp.splits = static_cast<int>(s);
  // Counters first, at a fixed place whatever the shape (a larger shape's partials must
  // never land on a later call's counters), then the partials.
  sp.cnt_offset = 0;
  sp.part_bytes = static_cast<size_t>(tiles) * 2 * s * kBM * kBN * sizeof(float);
  sp.bytes = kSplitCounterBytes + sp.part_bytes;
  return sp;
}

int units_for(int64_t m) {
  const int sms = sm_count();
  return m > kBM ? sms / 2 : sms;
}

template <bool kDual>
int run(const char* name, const void* x, int64_t ldx, const void* w, int64_t ldw,
        const void* w2, int64_t ldw2, const void* bias, const void* residual, int64_t ldr,
        void* y, int64_t ldy, int64_t m, int64_t n, int64_t k, int epilogue, void* stream,
        void* workspace = nullptr, size_t workspace_bytes = 0) {
  clear_error();
  if (m < 0 || n < 0 || k <= 0) return fail(UMIC_ERR_INVALID_ARG, "%s: bad sizes", name);
  if (m == 0 || n == 0) return UMIC_OK;
  if (m > 0x7fffffffLL - kBM || n > 0x7fffffffLL - kBN || k > 0x7fffffffLL)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: size too large", name);
  if (k % 8) return fail(UMIC_ERR_ALIGNMENT, "%s: k=%lld not a multiple of 8", name,
                         (long long)k);
  if (n % 8) return fail(UMIC_ERR_UNSUPPORTED, "%s: n=%lld not a multiple of 8", name,
                         (long long)n);
  if (int rc = check_operand(name, "x", x, ldx, k)) return rc;
  if (int rc = check_operand(name, "w", w, ldw, k)) return rc;
  if (kDual)
    if (int rc = check_operand(name, "w_up", w2, ldw2, k)) return rc;
  if (!y || !aligned16(y) || ldy % 8 || ldy < n)
    return fail(UMIC_ERR_ALIGNMENT, "%s: output must be 16-byte aligned with ld %% 8 == 0", name);
  if (bias && !aligned16(bias)) return fail(UMIC_ERR_ALIGNMENT, "%s: bias alignment", name);
  if (residual && (!aligned16(residual) || ldr % 8 || ldr < n))
    return fail(UMIC_ERR_ALIGNMENT, "%s: residual alignment", name);
  if (epilogue < UMIC_EPI_NONE || epilogue > UMIC_EPI_GELU_TANH)
    return fail(UMIC_ERR_INVALID_ARG, "%s: bad epilogue %d", name, epilogue);

  const int out_cols = kDual ? kBN / 2 : kBN;
  // A CTA pair (256-row tiles) whenever there is more than one 128-row block.
  const bool pair = m > kBM;
  const int b_rows = pair ? kBN / 2 : (kDual ? kBN / 2 : kBN);
  CUtensorMap ma, mb, mb2, my;
  if (!make_out_map(&my, y, m, n, ldy))
    return fail(UMIC_ERR_DEVICE, "%s: output tensor map rejected", name);
  if (!make_map(&ma, x, m, k, ldx, kBM) || !make_map(&mb, w, n, k, ldw, b_rows) ||
      !make_map(&mb2, kDual ? w2 : w, n, k, kDual ? ldw2 : ldw, b_rows))
    return fail(UMIC_ERR_DEVICE, "%s: cuTensorMapEncodeTiled unavailable or rejected", name);

  TcParams p;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.ldy = ldy;
  p.ldr = ldr;
  p.err = device_error_word();
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  const int tile_m = pair ? 2 * kBM : kBM;
  p.tiles_m = static_cast<int>((m + tile_m - 1) / tile_m);
  p.tiles_n = static_cast<int>((n + out_cols - 1) / out_cols);
  p.kblocks = static_cast<int>((k + kBK - 1) / kBK);
  p.epilogue = epilogue;
  p.splits = 1;
  p.part = nullptr;
  p.cnt = nullptr;
  if (!kDual && workspace) {
    const SplitPlan sp = plan_split(m, n, k, units_for(m));
    if (sp.splits > 1) {
      if (workspace_bytes < sp.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return fail(UMIC_ERR_INVALID_ARG, "%s: workspace of %zu bytes (256-byte aligned) "
                    "needed, %zu given", name, sp.bytes, workspace_bytes);
      p.splits = sp.splits;
      p.cnt = static_cast<unsigned*>(workspace);
      p.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kSplitCounterBytes);
    }
  }
  p.wait_limit = kWaitLimitCycles;
  p.stall = 0;
  {
    long long limit = 0;
    if (take_stall(kStallGemm, &limit)) {
      p.stall = 1;
      p.wait_limit = limit;
    }
  }
  const int64_t tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n * p.splits;  // work units
  if (tiles > 0x7fffffffLL) return fail(UMIC_ERR_UNSUPPORTED, "%s: too many tiles", name);
  const int sms = sm_count();
  cudaStream_t st = as_stream(stream);
  if (!pair) {
    if (int rc = set_smem_attr<kDual, 1>()) return rc;
    const int grid = static_cast<int>(tiles < sms ? tiles : sms);
    const cudaError_t le = launch_pdl(tc_gemm_kernel<kDual, 1>, dim3(grid), dim3(kThreads),
                                      Geo<1>::kSmem, st, ma, mb, mb2, my, p);
    if (le != cudaSuccess) return fail(UMIC_ERR_LAUNCH, "%s: %s", name, cudaGetErrorString(le));
    return launch_status(name);
  }
  if (int rc = set_smem_attr<kDual, 2>()) return rc;
  const int pairs = static_cast<int>(tiles < sms / 2 ? tiles : sms / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Geo<2>::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // programmatic stream serialization: see the grid dependency wait in the kernel
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, tc_gemm_kernel<kDual, 2>, ma, mb, mb2, my, p);
  if (e != cudaSuccess) return fail(UMIC_ERR_LAUNCH, "%s: %s", name, cudaGetErrorString(e));
  return launch_status(name);
}

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" {

int umic_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
              const void* residual, int64_t ldr, void* y, int64_t ldy, int64_t m, int64_t n,
              int64_t k, int epilogue, void* stream) {
  return run<false>("umic_gemm", x, ldx, w, ldw, nullptr, 0, bias, residual, ldr, y, ldy, m, n, k,
                    epilogue, stream);
}

int umic_gemm_ws(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
                 const void* residual, int64_t ldr, void* y, int64_t ldy, int64_t m, int64_t n,
                 int64_t k, int epilogue, void* workspace, size_t workspace_bytes,
                 void* stream) {
  return run<false>("umic_gemm_ws", x, ldx, w, ldw, nullptr, 0, bias, residual, ldr, y, ldy, m,
                    n, k, epilogue, stream, workspace, workspace_bytes);
}

size_t umic_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return plan_split(m, n, k, units_for(m)).bytes;
}

int umic_gemm_gate_silu_mul(const void* x, int64_t ldx, const void* wg, int64_t ldwg,
                            const void* wu, int64_t ldwu, void* h, int64_t ldh, int64_t m,
                            int64_t n, int64_t k, void* stream) {
  return run<true>("umic_gemm_gate_silu_mul", x, ldx, wg, ldwg, wu, ldwu, nullptr, nullptr, 0, h,
                   ldh, m, n, k, UMIC_EPI_NONE, stream);
}

}  // extern "C"
