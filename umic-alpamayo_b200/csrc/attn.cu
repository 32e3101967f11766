// Attention of a few query rows per KV head over a long key/value prefix, on the
// tcgen05 tensor cores (TMEM accumulators, TMA-fed shared memory).
//
// The shape is the flow expert's Euler step: T action tokens whose G query heads
// share one KV head (G * T <= 128 rows) attend over Lk cached keys under a boolean
// mask (transformers' causal mask of the new tokens over the cache), given as bits
// (umic_mask_pack_bits packs the boolean mask: one 32-bit word per 32 keys, so a
// thread reads two words per block instead of 64 scattered bytes). One CTA per
// (batch, kv head) holds its G * T query rows as one M = 128 tile and streams the
// keys and values through a 5-stage ring of 64-key blocks. Per block:
//   S = Q K^T               tcgen05.mma M128 N64 K128 into TMEM (K-major operands);
//   P = exp2(S' - m)        eight warps, two per query row: each thread takes 32
//                           of a row's 64 keys (the pair swaps row maxima through
//                           shared memory), keeps the running max m (online
//                           softmax), rounds P to bf16 and writes it over the
//                           block's K slot (the K block is dead once S is
//                           computed); the running sum l adds the rounded values,
//                           so the weights applied to V sum to 1;
//   O = alpha * O + P V     O accumulates in TMEM across blocks; V is the
//                           MN-major operand (d contiguous), so no transpose is
//                           made; O is rescaled in place only in warps whose
//                           running max moved (after the first blocks, almost none).
// The MMA for S of block j+1 runs while the softmax warps work on block j.
// At the end each thread divides its row by l and writes it as bf16.
//
// HBM-bound at the flow shape (every K/V byte is read once: 415 MB per layer for
// 32 episodes x 8 KV heads x 3164 keys): one CTA per SM keeps 160 KB of K/V in
// flight (a 2-stage ring at two CTAs per SM left each block waiting on its load),
// and two softmax warps per SM sub-partition hide each other's latencies.
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
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 softmax
constexpr uint32_t kQBytes = kRows * kD * 2;          // 32 KB: two 16 KB atom columns
constexpr uint32_t kKBytes = kKeys * kD * 2;          // 16 KB: two 8 KB atom columns
constexpr uint32_t kStageBytes = 2 * kKBytes;         // K (later P) + V
constexpr uint32_t kBarOff = kQBytes + kStages * kStageBytes;
constexpr uint32_t kXchOff = kBarOff + 256;          // row maxima / sums exchanged
constexpr size_t kSmem = kXchOff + 2 * 2 * kRows * 4 + 1024;  // [parity][half][row], align
constexpr uint32_t kTmemCols = 256;                   // S: cols 0-63, O: cols 128-255
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
  // q_full, kv_full[kStages], kv_empty[kStages], s_full, s_empty, p_full, o_full, drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6 + 2 * kStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t q_full = smem_u32(bars), kv_full0 = q_full + 8;
  const uint32_t kv_empty0 = kv_full0 + 8 * kStages, s_full = kv_empty0 + 8 * kStages;
  const uint32_t s_empty = s_full + 8, p_full = s_full + 16, o_full = s_full + 24;
  const uint32_t drain = s_full + 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / p.hkv, h = blockIdx.x % p.hkv;
  const uint32_t qs = sbase;
  auto kslot = [&](int s) { return sbase + kQBytes + s * kStageBytes; };
  auto vslot = [&](int s) { return sbase + kQBytes + s * kStageBytes + kKBytes; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(kv_full0 + 8 * s, 1);
      mbar_init(kv_empty0 + 8 * s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 256);
    mbar_init(p_full, 256);
    mbar_init(o_full, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      // Q rows (g, t) -> tile row g * T + t; two 64-wide d halves (atom columns).
      mbar_expect_tx(q_full, static_cast<uint32_t>(p.g * p.t) * kD * 2);
      for (int g = 0; g < p.g; ++g)
        for (int half = 0; half < 2; ++half)
          tma_load_4d(qs + half * (kQBytes / 2) + g * p.t * 128, &map_q, q_full, half * 64,
                      h * p.g + g, 0, b);
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
      const uint32_t tmem_s = tmem_base, tmem_o = tmem_base + kTmemO;
      auto issue_s = [&](int s) {
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          // d step of 16 = 32 bytes inside an atom column; columns are 16 KB (Q) / 8 KB (K) apart
          const uint32_t qa = qs + (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32;
          const uint32_t ka = kslot(s) + (kk >> 2) * (kKBytes / 2) + (kk & 3) * 32;
          mma(tmem_s, sdesc(qa, 16, 1024), sdesc(ka, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, p.err, abort_flag) &&
                mbar_wait(kv_full0, 0, p.err, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        commit(s_full);
      }
      for (int j = 0; ok && j < p.nblk; ++j) {
        const int s = j % kStages;
        if (j + 1 < p.nblk) {
          // S of the next block as soon as its keys are in and S_j has been read.
          const int s1 = (j + 1) % kStages;
          if (!mbar_wait(kv_full0 + 8 * s1, ((j + 1) / kStages) & 1, p.err, abort_flag) ||
              !mbar_wait(s_empty, j & 1, p.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(s1);
          commit(s_full);
        }
        if (!mbar_wait(p_full, j & 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          // P: one 128-row atom column, key step of 16 = 32 bytes. V (MN-major): key
          // step of 16 = two 8-key groups of 1024 bytes; d halves 8 KB apart.
          const uint32_t pa = kslot(s) + kk * 32;
          const uint32_t va = vslot(s) + kk * 2048;
          mma(tmem_o, sdesc(pa, 16, 1024), sdesc(va, kKBytes / 2, 1024), kIdescPV,
              (j > 0 || kk > 0) ? 1u : 0u);
        }
        commit(o_full);
        commit(kv_empty0 + 8 * s);  // K/P and V slots free for block j + kStages
      }
      commit(drain);
      mbar_wait(drain, 0, p.err, abort_flag);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- softmax
    // Warps w and w + 4 share TMEM lanes 32 * (w % 4), i.e. 32 query rows: half 0
    // takes keys 0-31 of each block and O columns 0-63, half 1 keys 32-63 and O
    // columns 64-127. Both pass or fail the same waits, so neither is left alone
    // at their named barrier.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const bool valid = r < p.g * p.t;
    const int g = valid ? r / p.t : 0, t = valid ? r % p.t : 0;
    const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t ts = tmem_base + lanes + 32 * half;
    const uint32_t to = tmem_base + lanes + kTmemO + 64 * half;
    float* xch = reinterpret_cast<float*>(smem + kXchOff);  // [parity][half][row]
    const uint32_t pair_bar = 1 + quarter;
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory"); };
    const uint32_t* mrow =
        p.bits ? p.bits + b * p.m_sb + (h * p.g + g) * p.m_sh + t * p.m_st : nullptr;
    const int words = (p.lk + 31) >> 5;
    // this block's mask word (keys 32 * half .. + 31), loaded one block ahead
    uint32_t w = 0xffffffffu;
    if (mrow && valid) w = half < words ? __ldg(mrow + half) : 0u;
    const float ninf = -INFINITY, sl2 = p.scale_log2;
    float m_run = ninf, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < p.nblk; ++j) {
      if (!mbar_wait(s_full, j & 1, p.err, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[32];
      tmem_ld32(ts, sv);
      tc_fence_before();
      mbar_arrive(s_empty);
      // keys past Lk are cut by index (their bits, if any, are padding)
      const int left = p.lk - (j * kKeys + 32 * half);
      const uint32_t lim = left >= 32 ? 0xffffffffu : (left > 0 ? (1u << left) - 1u : 0u);
      const uint32_t mw = valid ? (w & lim) : 0u;
      if (mrow && valid) {
        const int wi = 2 * j + 2 + half;
        w = wi < words ? __ldg(mrow + wi) : 0u;
      }
      if (!__all_sync(0xffffffffu, mw == 0xffffffffu)) {  // masked keys in this warp's block
#pragma unroll
        for (int c = 0; c < 32; ++c) sv[c] = (mw >> c) & 1u ? sv[c] : ninf;
      }
      // tree reductions keep the dependent chains short
      float mx[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) mx[c] = fmaxf(sv[c], sv[c + 16]);
#pragma unroll
      for (int w2 = 8; w2 >= 1; w2 >>= 1)
#pragma unroll
        for (int c = 0; c < w2; ++c) mx[c] = fmaxf(mx[c], mx[c + w2]);
      float mb = mx[0];
      float* xj = xch + (j & 1) * 2 * kRows;
      xj[half * kRows + r] = mb;
      pair_sync();
      mb = fmaxf(mb, xj[(half ^ 1) * kRows + r]);
      // raw scores are scaled inside the exponent: p = 2^(s * scale * log2 e - m')
      const float m_new = fmaxf(m_run, mb);
      const float m_use = m_new == ninf ? 0.f : m_new;
      const float alpha = ex2((m_run - m_use) * sl2);
      const float msc = m_use * sl2;
      float ps[16];
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const __nv_bfloat162 pb = __floats2bfloat162_rn(ex2(fmaf(sv[c], sl2, -msc)),
                                                        ex2(fmaf(sv[c + 1], sl2, -msc)));
        // the row sum of the rounded weights the MMA uses, so they sum to exactly 1
        const float2 f = __bfloat1622float2(pb);
        ps[c / 2] = f.x + f.y;
        pk[c / 2] = *reinterpret_cast<const uint32_t*>(&pb);
      }
#pragma unroll
      for (int w2 = 8; w2 >= 1; w2 >>= 1)
#pragma unroll
        for (int c = 0; c < w2; ++c) ps[c] += ps[c + w2];
      l_run = l_run * alpha + ps[0];  // this half's share of the row sum
      m_run = m_new;
      if (j > 0) {
        // O holds blocks < j at the old max: wait for P_{j-1} V_{j-1}, then rescale
        // this warp's 64 columns if some row's max moved.
        if (!mbar_wait(o_full, (j - 1) & 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < 64; c += 32) {
            float o[32];
            tmem_ld32(to + c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(to + c, o);
          }
        }
      }
      // P_j over this block's K slot: row r, 16-byte chunk c8 at r * 128 + (c8 ^ (r & 7)) * 16;
      // this half writes chunks 4 * half .. 4 * half + 3.
      const uint32_t pbase = kslot(j % kStages) + r * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        st_shared_v4(pbase + (((4 * half + i) ^ (r & 7)) << 4),
                     make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]));
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(o_full, (p.nblk - 1) & 1, p.err, abort_flag)) {
      tc_fence_after();
      // whole-row sum: the two halves meet in the exchange buffer the last block left free
      float* xl = xch + (p.nblk & 1) * 2 * kRows;
      xl[half * kRows + r] = l_run;
      pair_sync();
      const float l = l_run + xl[(half ^ 1) * kRows + r];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow =
          p.out + b * p.o_sb + (h * p.g + g) * p.o_sh + t * p.o_st + 64 * half;
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        float o[32];
        tmem_ld32(to + c, o);
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float f[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) f[jj] = o[i + jj] * inv;
            st_vec(orow + c + i, pack8(f));
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
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int ti = static_cast<int>(row % t);
  const int64_t rest = row / t;
  const int hi = static_cast<int>(rest % hm);
  const int64_t bi = rest / hm;
  const uint8_t* src = mask + bi * sb + hi * sh + ti * st;
  uint32_t* dst = bits + bi * wb + hi * wh + ti * wt;
  for (int w = 0; w < (lk + 31) >> 5; ++w) {
    const int key = w * 32 + lane;
    const uint32_t word = __ballot_sync(0xffffffffu, key < lk && src[key] != 0);
    if (lane == 0) dst[w] = word;
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
  if (d != kD) return fail(UMIC_ERR_UNSUPPORTED, "%s: head_dim %lld (128 only)", kName,
                           (long long)d);
  if (hq % hkv) return fail(UMIC_ERR_UNSUPPORTED, "%s: %lld query heads over %lld kv heads",
                            kName, (long long)hq, (long long)hkv);
  const int64_t g = hq / hkv;
  if (!(scale > 0.f)) return fail(UMIC_ERR_INVALID_ARG, "%s: scale must be positive", kName);
  if (g * t > kRows || t % 8 || lk < 1)
    return fail(UMIC_ERR_UNSUPPORTED,
                "%s: %lld query rows per kv head (<= 128, tokens a multiple of 8, keys >= 1)",
                kName, (long long)(g * t));
  if (batch * hkv > 0x7fffffffLL || lk > 0x7fffffffLL - kKeys)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: size too large", kName);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !stride_ok(q_sh) ||
      !stride_ok(q_st) || !stride_ok(q_sb) || !stride_ok(k_sl) || !stride_ok(k_sh) ||
      !stride_ok(k_sb) || !stride_ok(v_sl) || !stride_ok(v_sh) || !stride_ok(v_sb) ||
      o_sb % 8 || o_sh % 8 || o_st % 8)
    return fail(UMIC_ERR_ALIGNMENT, "%s: 16-byte aligned bases and strides required", kName);
  if (mask_bits && (m_sb < 0 || m_sh < 0 || m_st < 0))
    return fail(UMIC_ERR_INVALID_ARG, "%s: negative mask stride", kName);
  CUtensorMap mq, mk, mv;
  // q as (d, head, token, batch); k / v as (d, key, kv head, batch)
  if (!make_map4(&mq, q, kD, hq, t, batch, q_sh, q_st, q_sb, 1, static_cast<int>(t)) ||
      !make_map4(&mk, k, kD, lk, hkv, batch, k_sl, k_sh, k_sb, kKeys, 1) ||
      !make_map4(&mv, v, kD, lk, hkv, batch, v_sl, v_sh, v_sb, kKeys, 1))
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
  attn_rows_kernel<<<static_cast<unsigned>(batch * hkv), kThreads, kSmem, as_stream(stream)>>>(
      mq, mk, mv, p);
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
  mask_pack_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(mask), sb, sh, st, static_cast<int>(heads), static_cast<int>(t),
      static_cast<int>(lk), bits, wb, wh, wt, rows);
  return launch_status(kName);
}
