// Attention of a few query rows per KV head over a long key/value prefix, on the
// tcgen05 tensor cores (TMEM accumulators, TMA-fed shared memory).
//
// The shape is the flow expert's Euler step: T action tokens whose G query heads
// share one KV head (G * T <= 128 rows) attend over Lk cached keys under a boolean
// mask (transformers' causal mask of the new tokens over the cache), given as bits
// (umic_mask_pack_bits packs the boolean mask: one 32-bit word per 32 keys, so a
// thread reads two words per block instead of 64 scattered bytes). One CTA per
// (batch, kv head) holds its G * T query rows as one M = 128 tile and streams the
// keys and values through a 5-stage ring of 64-key blocks. Per block j:
//   S = Q K^T               tcgen05.mma M128 N64 K128 into TMEM (K-major operands);
//   P = exp2(S' - m)        softmax warp group j % 2, one query row per thread:
//                           mask, scale, running max m and sum l of the group's
//                           blocks (online softmax), P rounded to bf16 and written
//                           over the block's K slot (the K block is dead once S is
//                           computed); l adds the rounded values, so the weights
//                           applied to V sum to 1;
//   O_g = alpha O_g + P V   into the group's own TMEM accumulator (V is the
//                           MN-major operand, d contiguous, so no transpose is
//                           made); the reference max moves, and O_g is rescaled
//                           in place, only when a row's max grows by more than 8
//                           in log2 units (weights stay <= 256), i.e. rarely.
// The two groups (warps 2-5 and 6-9, one of each on every SM sub-partition) run
// independent chains on alternate blocks and exchange nothing until the end, where
// each row's two partial results are merged with their maxima and sums. With one
// query head per KV head, longer token ranges are cut into 128-row tiles, one CTA each
// (the ViT: 1024 patches per image and head); head dims below 128 (the ViT's 80) are
// zero-filled by TMA, which adds nothing to S or O. The MMA
// for S of block j + 2 is issued as soon as group j % 2 has read S of block j, so
// it runs while the group works on block j.
//
// Every K/V byte is read once (415 MB per layer for 32 episodes x 8 KV heads x 3164
// keys at the flow shape). A slot of the ring is refilled only after the P V of its
// block, and a block's load takes ~3 us to land under this traffic, so each slot
// turns over about every 5 us: the ring, not HBM, sets the pace (about 1 us per
// block per CTA, 0.5-0.6 of the HBM bound; six stages or an L2 prefetch of each slot's
// next block measured no faster).
//
// Every mbarrier wait is bounded; a wait that runs out sets
// UMIC_DEVERR_WAIT_TIMEOUT, the CTA lets its copies land, drains its MMAs, frees
// TMEM and exits.
#include <cuda.h>

#include <cmath>
#include <mutex>

#include "common.cuh"
#include "tma.cuh"

namespace umic {
namespace {

constexpr int kD = 128;        // head dim
constexpr int kRows = 128;     // query rows per CTA (TMEM lanes)
constexpr int kKeys = 64;      // keys per block
constexpr int kStages = 5;
// S of block j + 2 is issued before P V of block j, whose stage the ring refills:
// with fewer than three stages the ring could not hold block j + 2 yet.
static_assert(kStages >= 3, "the MMA issuer runs two blocks ahead of the P V MMAs");
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 softmax
constexpr uint32_t kQBytes = kRows * kD * 2;          // 32 KB: two 16 KB atom columns
constexpr uint32_t kKBytes = kKeys * kD * 2;          // 16 KB: two 8 KB atom columns
constexpr uint32_t kStageBytes = 2 * kKBytes;         // K (later P) + V
constexpr uint32_t kBarOff = kQBytes + kStages * kStageBytes;
constexpr size_t kSmem = kBarOff + 256 + 1024;        // barriers and flags, alignment
constexpr uint32_t kTmemCols = 512;  // S_0, S_1: cols 0-63, 64-127; O_0, O_1: 128-255, 256-383
constexpr uint32_t kTmemO = 128;

// kind::f16 instruction descriptors: D fp32, A/B bf16, M = 128.
//   S = Q K^T: N = 64, both operands K-major.
//   O += P V: N = 128, A (P) K-major, B (V) MN-major (bit 16).
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) |
                             ((128u >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) |
                              ((128u >> 3) << 17) | ((128u >> 4) << 24);

struct AttnParams {
  const uint32_t* bits;     // mask bits [B, Hm, T, ceil(Lk / 32)] (key k: bit k % 32 of word k / 32), or null
  int64_t m_sb, m_sh, m_st; // word strides; 0 broadcasts
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_st;
  uint32_t* err;
  int hq, hkv, g, t, lk, nblk;
  int qtiles;  // > 1: one query head per KV head, rows t0 .. t0 + 127 per CTA (t0 = 128 qt)
  int d;       // head dim (<= 128; the tiles are zero-filled past it)
  float scale_log2;         // softmax scale * log2(e)
};

// Shared-memory matrix descriptor, 128-byte swizzle, version 1 (sm_100).
// K-major: SBO = 1024 (8-row groups), LBO unused. MN-major: LBO = distance between
// the 64-element atoms along MN, SBO = distance between 8-row groups along K.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t ad, uint64_t bd, uint32_t idesc,
                                    uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(ad), "l"(bd), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                   "r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 consecutive fp32 columns; thread i gets lane (base + i).
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

// 32 lanes x 64 consecutive fp32 columns in one load and one wait (the softmax reads a
// whole block's scores per thread; two 32-column loads would pay two round trips).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2^x on the special-function unit; results below the normal range flush to zero
// (attention weights that small contribute nothing at bf16).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Non-blocking check that the phase with the given parity has completed
// (mbarrier.try_wait may suspend the thread for a while when it has not, which would
// hold up the MMA issuer's other work).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void st_shared_v4(uint32_t a, const uint4& v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_rows_kernel(const __grid_constant__ CUtensorMap map_q,
                     const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  // q_full, kv_full[kStages], kv_empty[kStages], s_full[2], s_empty[2], p_full[2][2],
  // o_full[2], o_last, drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13 + 2 * kStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t q_full = smem_u32(bars), kv_full0 = q_full + 8;
  const uint32_t kv_empty0 = kv_full0 + 8 * kStages, s_full = kv_empty0 + 8 * kStages;
  // Per softmax group g: s_full[g] (S of its next block is in TMEM), s_empty[g] (the
  // group has read it), p_full[g][n & 1] (P of the group's n-th block is in shared
  // memory; two barriers, as the group may finish its next block before the issuer
  // looks), o_full[g] (P V of its block landed in O_g). o_last: every MMA done (the
  // final read of O_0 and O_1).
  const uint32_t s_empty0 = s_full + 16, p_full0 = s_full + 32, o_full0 = s_full + 64;
  const uint32_t o_last = s_full + 80, drain = s_full + 88;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = static_cast<int>(blockIdx.x) % p.qtiles;
  const int bh = static_cast<int>(blockIdx.x) / p.qtiles;
  const int b = bh / p.hkv, h = bh % p.hkv;
  const int t0 = qt * kRows;
  const uint32_t qs = sbase;
  auto kslot = [&](int s) { return sbase + kQBytes + s * kStageBytes; };
  auto vslot = [&](int s) { return sbase + kQBytes + s * kStageBytes + kKBytes; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(kv_full0 + 8 * s, 1);
      mbar_init(kv_empty0 + 8 * s, 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full + 8 * g, 1);
      mbar_init(s_empty0 + 8 * g, 128);
      mbar_init(p_full0 + 16 * g, 128);
      mbar_init(p_full0 + 16 * g + 8, 128);
      mbar_init(o_full0 + 8 * g, 1);
    }
    mbar_init(o_last, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    prefetch_map(&map_q);
    prefetch_map(&map_k);
    prefetch_map(&map_v);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // set-up above overlaps the previous kernel's tail (launch_pdl); its outputs (q, the
  // KV cache, the mask bits) are read only after it has completed
  allow_dependent_launch();
  wait_prerequisite();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      // Q rows (g, t) -> tile row g * T + t (one tile), or t - t0 (tiled over tokens);
      // two 64-wide d halves (atom columns); d past the head dim arrives as zeros.
      if (p.qtiles == 1) {
        mbar_expect_tx(q_full, static_cast<uint32_t>(p.g * p.t) * kD * 2);
        for (int g = 0; g < p.g; ++g)
          for (int half = 0; half < 2; ++half)
            tma_load_4d(qs + half * (kQBytes / 2) + g * p.t * 128, &map_q, q_full, half * 64,
                        h * p.g + g, 0, b);
      } else {
        mbar_expect_tx(q_full, kQBytes);
        for (int half = 0; half < 2; ++half)
          tma_load_4d(qs + half * (kQBytes / 2), &map_q, q_full, half * 64, h, t0, b);
      }
      int j = 0;
      for (; j < p.nblk; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(kv_empty0 + 8 * s, ph ^ 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t fb = kv_full0 + 8 * s;
        mbar_expect_tx(fb, kStageBytes);  // keys past Lk arrive as zeros
        for (int half = 0; half < 2; ++half) {
          tma_load_4d(kslot(s) + half * (kKBytes / 2), &map_k, fb, half * 64, j * kKeys, h, b);
          tma_load_4d(vslot(s) + half * (kKBytes / 2), &map_v, fb, half * 64, j * kKeys, h, b);
        }

      }
      if (ok) {
        // The last stages are released by the MMA before the CTA may exit.
        for (int jj = j > kStages ? j - kStages : 0; jj < j; ++jj)
          if (!mbar_wait(kv_empty0 + 8 * (jj % kStages), (jj / kStages) & 1, p.err, abort_flag))
            break;
      } else {
        const long long t0 = clock64();  // let copies in flight land
        while (clock64() - t0 < 4000000LL) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      auto issue_s = [&](int s, int g) {
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          // d step of 16 = 32 bytes inside an atom column; columns are 16 KB (Q) / 8 KB (K) apart
          const uint32_t qa = qs + (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32;
          const uint32_t ka = kslot(s) + (kk >> 2) * (kKBytes / 2) + (kk & 3) * 32;
          mma(tmem_base + 64 * g, sdesc(qa, 16, 1024), sdesc(ka, 16, 1024), kIdescS,
              kk > 0 ? 1u : 0u);
        }
        commit(s_full + 8 * g);
      };
      auto kv_ready = [&](int j) {
        return mbar_wait(kv_full0 + 8 * (j % kStages), (j / kStages) & 1, p.err, abort_flag);
      };
      bool ok = mbar_wait(q_full, 0, p.err, abort_flag);
      for (int j = 0; ok && j < 2 && j < p.nblk; ++j) {
        ok = kv_ready(j);
        if (ok) {
          tc_fence_after();
          issue_s(j % kStages, j);
        }
      }
      // Event loop: issue whichever is ready -- S of block ns (its group has read S of
      // block ns - 2, its keys are in) or P V of block npv (its group wrote P) -- so
      // neither group waits behind the other. S runs at most three blocks ahead of P V
      // (ns < npv + 4), so a group can be at most one of its own blocks past the one
      // whose P this thread waits for (hence two p_full barriers per group), and every
      // other barrier at most at the phase waited for: every parity wait stays exact.
      int ns = p.nblk < 2 ? p.nblk : 2, npv = 0;
      const long long t0 = clock64();
      for (uint32_t spin = 0; ok && npv < p.nblk;) {
        bool progressed = false;
        if (ns < p.nblk && ns < npv + 4) {
          const int g = ns & 1, n = (ns - 2) >> 1;
          if (mbar_test(s_empty0 + 8 * g, n & 1) &&
              mbar_test(kv_full0 + 8 * (ns % kStages), (ns / kStages) & 1)) {
            tc_fence_after();
            issue_s(ns % kStages, g);
            ++ns;
            progressed = true;
          }
        }
        {
          const int g = npv & 1, s = npv % kStages, n = npv >> 1;
          if (mbar_test(p_full0 + 16 * g + 8 * (n & 1), (n >> 1) & 1)) {
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kKeys / 16; ++kk) {
              // P: one 128-row atom column, key step of 16 = 32 bytes. V (MN-major): key
              // step of 16 = two 8-key groups of 1024 bytes; d halves 8 KB apart.
              const uint32_t pa = kslot(s) + kk * 32;
              const uint32_t va = vslot(s) + kk * 2048;
              mma(tmem_base + kTmemO + 128 * g, sdesc(pa, 16, 1024),
                  sdesc(va, kKBytes / 2, 1024), kIdescPV, (npv >= 2 || kk > 0) ? 1u : 0u);
            }
            commit(o_full0 + 8 * g);
            commit(kv_empty0 + 8 * s);  // K/P and V slots free for block npv + kStages
            ++npv;
            progressed = true;
          }
        }
        if (progressed) {
          spin = 0;
        } else if ((++spin & 255u) == 0) {
          if (*abort_flag) {
            ok = false;
          } else if (clock64() - t0 > kWaitLimitCycles) {
            *abort_flag = 1;
            if (p.err) atomicOr(p.err, UMIC_DEVERR_WAIT_TIMEOUT);
            ok = false;
          }
        }
      }
      if (ok) commit(o_last);
      commit(drain);
      mbar_wait(drain, 0, p.err, abort_flag);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- softmax
    // Group g = warps 2-5 (g 0) or 6-9 (g 1) takes blocks j = g, g + 2, ...; warp w
    // reads TMEM lanes 32 * (w % 4), i.e. query rows 32 * (w % 4) .. + 31. Both
    // groups pass or fail the same final waits, so neither is left alone at the
    // named barrier where they merge.
    const int quarter = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const bool tiled = p.qtiles > 1;
    const bool valid = tiled ? t0 + r < p.t : r < p.g * p.t;
    const int g = (!tiled && valid) ? r / p.t : 0;
    const int t = tiled ? t0 + r : (valid ? r % p.t : 0);
    const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t ts = tmem_base + lanes + 64 * grp;
    const uint32_t to0 = tmem_base + lanes + kTmemO;  // O_0; O_1 is 128 columns on
    const uint32_t to = to0 + 128 * grp;
    const uint32_t* mrow =
        p.bits ? p.bits + b * p.m_sb + (h * p.g + g) * p.m_sh + t * p.m_st : nullptr;
    const int words = (p.lk + 31) >> 5;
    // the mask words of the group's current block, loaded one block ahead
    uint32_t w0 = 0xffffffffu, w1 = 0xffffffffu;
    if (mrow && valid) {
      w0 = 2 * grp < words ? __ldg(mrow + 2 * grp) : 0u;
      w1 = 2 * grp + 1 < words ? __ldg(mrow + 2 * grp + 1) : 0u;
    }
    const float ninf = -INFINITY, sl2 = p.scale_log2;
    float m_run = ninf, l_run = 0.f;
    bool ok = true;
    for (int j = grp, n = 0; j < p.nblk; j += 2, ++n) {
      if (!mbar_wait(s_full + 8 * grp, n & 1, p.err, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[64];
      tmem_ld64(ts, sv);
      float* s0 = sv;
      float* s1 = sv + 32;
      tc_fence_before();
      mbar_arrive(s_empty0 + 8 * grp);  // S_g may take the group's next block now
      // keys past Lk are cut by index (their bits, if any, are padding)
      const int left = p.lk - j * kKeys;
      const uint32_t lim0 = left >= 32 ? 0xffffffffu : (left > 0 ? (1u << left) - 1u : 0u);
      const uint32_t lim1 = left >= 64 ? 0xffffffffu : (left > 32 ? (1u << (left - 32)) - 1u : 0u);
      const uint32_t m0 = valid ? (w0 & lim0) : 0u, m1 = valid ? (w1 & lim1) : 0u;
      if (mrow && valid) {
        const int wi = 2 * (j + 2);
        w0 = wi < words ? __ldg(mrow + wi) : 0u;
        w1 = wi + 1 < words ? __ldg(mrow + wi + 1) : 0u;
      }
      if (!__all_sync(0xffffffffu, (m0 & m1) == 0xffffffffu)) {  // masked keys in this block
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          s0[c] = (m0 >> c) & 1u ? s0[c] : ninf;
          s1[c] = (m1 >> c) & 1u ? s1[c] : ninf;
        }
      }
      // tree reductions keep the dependent chains short
      float mx[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) mx[c] = fmaxf(s0[c], s1[c]);
#pragma unroll
      for (int w2 = 16; w2 >= 1; w2 >>= 1)
#pragma unroll
        for (int c = 0; c < w2; ++c) mx[c] = fmaxf(mx[c], mx[c + w2]);
      // Raw scores are scaled inside the exponent: p = 2^(s * scale * log2 e - m').
      // The reference max m' moves only when the block's max exceeds it by more than
      // 8 (in log2 units): below that the weights stay <= 256, and O and l share the
      // stale reference, so the final O / l is unchanged while O is rescaled far less
      // often.
      const bool move = m_run == ninf || (mx[0] - m_run) * sl2 > 8.f;
      const float m_new = move ? fmaxf(m_run, mx[0]) : m_run;
      const float m_use = m_new == ninf ? 0.f : m_new;
      const float alpha = move ? ex2((m_run - m_use) * sl2) : 1.f;
      const float msc = m_use * sl2;
      float ps[32];
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const __nv_bfloat162 pa = __floats2bfloat162_rn(ex2(fmaf(s0[c], sl2, -msc)),
                                                        ex2(fmaf(s0[c + 1], sl2, -msc)));
        const __nv_bfloat162 pb = __floats2bfloat162_rn(ex2(fmaf(s1[c], sl2, -msc)),
                                                        ex2(fmaf(s1[c + 1], sl2, -msc)));
        // the row sum of the rounded weights the MMA uses, so they sum to exactly 1
        const float2 fa = __bfloat1622float2(pa), fb = __bfloat1622float2(pb);
        ps[c / 2] = fa.x + fa.y;
        ps[16 + c / 2] = fb.x + fb.y;
        pk[c / 2] = *reinterpret_cast<const uint32_t*>(&pa);
        pk[16 + c / 2] = *reinterpret_cast<const uint32_t*>(&pb);
      }
#pragma unroll
      for (int w2 = 16; w2 >= 1; w2 >>= 1)
#pragma unroll
        for (int c = 0; c < w2; ++c) ps[c] += ps[c + w2];
      l_run = l_run * alpha + ps[0];
      m_run = m_new;
      if (n > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // O_g holds the group's earlier blocks at the old max: wait for the last of
        // them (phase n - 1 of o_full[g]), then rescale. Without a rescale the wait is
        // skipped. S_j was issued after the P V of block j - 4 (S stays less than four
        // blocks ahead of P V), so s_full already implies phase n - 2 completed, and
        // block j's own P V is not issued yet: o_full[g] is at phase n - 1 or just past
        // it, never further.
        if (!mbar_wait(o_full0 + 8 * grp, (n - 1) & 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < kD; c += 32) {
          float o[32];
          tmem_ld32(to + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(to + c, o);
        }
      }
      // P_j over this block's K slot: row r, 16-byte chunk c8 at r * 128 + (c8 ^ (r & 7)) * 16.
      const uint32_t pbase = kslot(j % kStages) + r * 128;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        st_shared_v4(pbase + ((c8 ^ (r & 7)) << 4),
                     make_uint4(pk[4 * c8], pk[4 * c8 + 1], pk[4 * c8 + 2], pk[4 * c8 + 3]));
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_full0 + 16 * grp + 8 * (n & 1));
    }
    if (ok && mbar_wait(o_last, 0, p.err, abort_flag)) {
      tc_fence_after();
      // merge the two groups' partial rows: common max, weights, whole-row sum (the
      // exchange uses stage 0's K slot: every load and MMA has completed by now)
      float* xm = reinterpret_cast<float*>(smem + kQBytes);  // [group][row]
      float* xl = xm + 2 * kRows;
      xm[grp * kRows + r] = m_run;
      xl[grp * kRows + r] = l_run;
      asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
      const float ma = xm[r], mb2 = xm[kRows + r];
      const float mm = fmaxf(ma, mb2);
      const float mu = mm == ninf ? 0.f : mm;
      const float sa = ex2((ma - mu) * sl2), sb = ex2((mb2 - mu) * sl2);
      const float l = xl[r] * sa + xl[kRows + r] * sb;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool two = p.nblk > 1;  // O_1 holds data only if group 1 had a block
      __nv_bfloat16* orow = p.out + b * p.o_sb + (h * p.g + g) * p.o_sh + t * p.o_st + 64 * grp;
#pragma unroll 1
      for (int c = 64 * grp; c < 64 * grp + 64; c += 32) {
        float oa[32], ob[32];
        tmem_ld32(to0 + c, oa);
        if (two) {
          tmem_ld32(to0 + 128 + c, ob);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ob[i] = 0.f;
        }
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            if (c + i >= p.d) break;  // columns past the head dim are padding
            float f[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
              f[jj] = (oa[i + jj] * sa + ob[i + jj] * sb) * inv;
            st_vec(orow + (c - 64 * grp) + i, pack8(f));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols));
  }
}

// One warp per mask row: lane l reads byte 32 w + l of the row (a coalesced 32-byte
// read) and the warp's ballot is word w of the row's bits.
__global__ void __launch_bounds__(256) mask_pack_kernel(const uint8_t* __restrict__ mask,
                                                        int64_t sb, int64_t sh, int64_t st,
                                                        int hm, int t, int lk,
                                                        uint32_t* __restrict__ bits,
                                                        int64_t wb, int64_t wh, int64_t wt,
                                                        int64_t rows) {
  allow_dependent_launch();
  wait_prerequisite();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int ti = static_cast<int>(row % t);
  const int64_t rest = row / t;
  const int hi = static_cast<int>(rest % hm);
  const int64_t bi = rest / hm;
  const uint8_t* src = mask + bi * sb + hi * sh + ti * st;
  uint32_t* dst = bits + bi * wb + hi * wh + ti * wt;
  const int words = (lk + 31) >> 5;
  for (int w0 = 0; w0 < words; w0 += 8) {
    uint8_t v[8];  // eight independent loads in flight before the ballots
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int key = (w0 + i) * 32 + lane;
      v[i] = key < lk ? src[key] : 0;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t word = __ballot_sync(0xffffffffu, v[i] != 0);
      if (lane == 0 && w0 + i < words) dst[w0 + i] = word;
    }
  }
}

// 4-D bf16 tensor map (d, a, c, e) with element strides (1, s1, s2, s3): boxes of
// 64 d x box1 x box2 x 1, 128-byte swizzle, out-of-range elements read as zero.
bool make_map4(CUtensorMap* map, const void* base, int64_t n0, int64_t n1, int64_t n2, int64_t n3,
               int64_t s1, int64_t s2, int64_t s3, int box1, int box2) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(n0), static_cast<cuuint64_t>(n1),
                              static_cast<cuuint64_t>(n2), static_cast<cuuint64_t>(n3)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(s1) * 2, static_cast<cuuint64_t>(s2) * 2,
                                 static_cast<cuuint64_t>(s3) * 2};
  const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box1), static_cast<cuuint32_t>(box2), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool stride_ok(int64_t s) { return s > 0 && s % 8 == 0; }

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" int umic_attention_rows(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                                   const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sl,
                                   const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sl,
                                   const uint32_t* mask_bits, int64_t m_sb, int64_t m_sh,
                                   int64_t m_st,
                                   void* out, int64_t o_sb, int64_t o_sh, int64_t o_st,
                                   int64_t batch, int64_t hq, int64_t hkv, int64_t t, int64_t lk,
                                   int64_t d, float scale, void* stream) {
  static const char* kName = "umic_attention_rows";
  clear_error();
  if (batch < 0 || hq <= 0 || hkv <= 0 || t < 0 || lk < 0 || d <= 0)
    return fail(UMIC_ERR_INVALID_ARG, "%s: bad sizes", kName);
  if (batch == 0 || t == 0) return UMIC_OK;
  if (!q || !k || !v || !out) return fail(UMIC_ERR_INVALID_ARG, "%s: null pointer", kName);
  if (d < 64 || d > kD || d % 8)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: head_dim %lld (64..128, a multiple of 8)", kName,
                (long long)d);
  if (hq % hkv) return fail(UMIC_ERR_UNSUPPORTED, "%s: %lld query heads over %lld kv heads",
                            kName, (long long)hq, (long long)hkv);
  const int64_t g = hq / hkv;
  if (!(scale > 0.f)) return fail(UMIC_ERR_INVALID_ARG, "%s: scale must be positive", kName);
  // One tile of g * t <= 128 rows per KV head, or (one query head per KV head) tiles of
  // 128 tokens.
  const bool one_tile = g * t <= kRows && t % 8 == 0;
  if ((!one_tile && g != 1) || lk < 1)
    return fail(UMIC_ERR_UNSUPPORTED,
                "%s: %lld query rows per kv head (<= 128 with tokens a multiple of 8, or "
                "one query head per kv head; keys >= 1)",
                kName, (long long)(g * t));
  const int64_t qtiles = one_tile ? 1 : (t + kRows - 1) / kRows;
  if (batch * hkv * qtiles > 0x7fffffffLL || lk > 0x7fffffffLL - kKeys || t > 0x7fffffffLL)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: size too large", kName);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !stride_ok(q_sh) ||
      !stride_ok(q_st) || !stride_ok(q_sb) || !stride_ok(k_sl) || !stride_ok(k_sh) ||
      !stride_ok(k_sb) || !stride_ok(v_sl) || !stride_ok(v_sh) || !stride_ok(v_sb) ||
      !stride_ok(o_sb) || !stride_ok(o_sh) || !stride_ok(o_st))
    return fail(UMIC_ERR_ALIGNMENT, "%s: 16-byte aligned bases and strides required", kName);
  if (mask_bits && (m_sb < 0 || m_sh < 0 || m_st < 0))
    return fail(UMIC_ERR_INVALID_ARG, "%s: negative mask stride", kName);
  CUtensorMap mq, mk, mv;
  // q as (d, head, token, batch); k / v as (d, key, kv head, batch)
  const int tbox = one_tile ? static_cast<int>(t) : kRows;
  if (!make_map4(&mq, q, d, hq, t, batch, q_sh, q_st, q_sb, 1, tbox) ||
      !make_map4(&mk, k, d, lk, hkv, batch, k_sl, k_sh, k_sb, kKeys, 1) ||
      !make_map4(&mv, v, d, lk, hkv, batch, v_sl, v_sh, v_sb, kKeys, 1))
    return fail(UMIC_ERR_DEVICE, "%s: cuTensorMapEncodeTiled unavailable or rejected", kName);
  AttnParams p;
  p.bits = mask_bits;
  p.m_sb = m_sb;
  p.m_sh = m_sh;
  p.m_st = m_st;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.o_st = o_st;
  p.err = device_error_word();
  p.hq = static_cast<int>(hq);
  p.hkv = static_cast<int>(hkv);
  p.g = static_cast<int>(g);
  p.t = static_cast<int>(t);
  p.lk = static_cast<int>(lk);
  p.nblk = static_cast<int>((lk + kKeys - 1) / kKeys);
  p.qtiles = static_cast<int>(qtiles);
  p.d = static_cast<int>(d);
  p.scale_log2 = scale * 1.4426950408889634f;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    e = cudaFuncSetAttribute(attn_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmem));
  });
  if (e != cudaSuccess)
    return fail(UMIC_ERR_LAUNCH, "%s: smem attribute: %s", kName, cudaGetErrorString(e));
  const dim3 grid(static_cast<unsigned>(batch * hkv * qtiles));
  const cudaError_t le =
      launch_pdl(attn_rows_kernel, grid, dim3(kThreads), kSmem, as_stream(stream), mq, mk, mv, p);
  if (le != cudaSuccess) return fail(UMIC_ERR_LAUNCH, "%s: %s", kName, cudaGetErrorString(le));
  return launch_status(kName);
}

extern "C" int umic_mask_pack_bits(const void* mask, int64_t sb, int64_t sh, int64_t st,
                                   int64_t batch, int64_t heads, int64_t t, int64_t lk,
                                   uint32_t* bits, int64_t wb, int64_t wh, int64_t wt,
                                   void* stream) {
  static const char* kName = "umic_mask_pack_bits";
  clear_error();
  if (batch < 0 || heads < 0 || t < 0 || lk < 0 || sb < 0 || sh < 0 || st < 0 || wb < 0 ||
      wh < 0 || wt < 0)
    return fail(UMIC_ERR_INVALID_ARG, "%s: bad sizes or strides", kName);
  const int64_t rows = batch * heads * t;
  if (rows == 0 || lk == 0) return UMIC_OK;
  if (!mask || !bits) return fail(UMIC_ERR_INVALID_ARG, "%s: null pointer", kName);
  if (heads > 0x7fffffffLL || t > 0x7fffffffLL || lk > 0x7fffffffLL - 32 ||
      rows > (int64_t{1} << 40))
    return fail(UMIC_ERR_UNSUPPORTED, "%s: size too large", kName);
  const int64_t blocks = (rows + 7) / 8;
  const cudaError_t le = launch_pdl(
      mask_pack_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, as_stream(stream),
      static_cast<const uint8_t*>(mask), sb, sh, st, static_cast<int>(heads), static_cast<int>(t),
      static_cast<int>(lk), bits, wb, wh, wt, rows);
  if (le != cudaSuccess) return fail(UMIC_ERR_LAUNCH, "%s: %s", kName, cudaGetErrorString(le));
  return launch_status(kName);
}
