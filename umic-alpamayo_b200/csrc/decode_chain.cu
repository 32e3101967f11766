// Decode chain: the dependent GEMVs of one decoder layer's decode step as the phases of
// ONE persistent kernel, with the small row-wise ops between them folded into the phase
// boundaries.
//
//   phase 0  o   = attn . W_o^T                       (plain GEMV)
//            tail: summed = o + residual; normed = RMSNorm(summed) * w_post
//   phase 1  h   = silu(normed . W_gate^T) * (normed . W_up^T)   (gated GEMV)
//   phase 2  out = h . W_down^T + summed              (GEMV, residual epilogue)
//
// Why one kernel: a decode step reads every weight once at m <= 16 rows, so each GEMV
// is HBM-bound, and as separate launches each pays a fixed ~6-8 us (launch, the first TMA
// round trip, the split-row-block merge) and the small norm kernel between them ~5-7 us,
// against 5-30 us of useful streaming. Here the weight stream never stops at a phase
// boundary: the producer warp of every CTA walks the units of all phases in order and
// keeps its 4-stage TMA ring full, so while the consumers wait for the rest of the grid
// to finish phase p (the data dependence), the first 128 KB of phase p + 1's weights are
// already landing in shared memory.
//
// Work split inside a phase is the streaming GEMV's (gemv.cu): 64-row x 256-column units
// (128 columns per matrix for gate/up) dealt to the CTAs as contiguous equal ranges; a row
// block split between CTAs is merged in the workspace by its last contributor, in CTA
// order. Between phases, a grid barrier: every CTA counts itself in (release) and waits
// for the count (acquire). A phase with a tail op has its last arriving CTA run the tail
// (one CTA; the tail touches m rows) and then release the others. All CTAs must be
// resident at once: the kernel is launched cooperatively. Every wait is bounded; on
// expiry the CTA sets UMIC_DEVERR_WAIT_TIMEOUT and unwinds (the workspace must then be
// zeroed before its next use). The last CTA of the final phase returns the barrier
// counters to zero, so a captured graph replays with the workspace clean.
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"
#include "mma_frag.cuh"
#include "tma.cuh"

namespace umic {
namespace {

constexpr int kRows = 64;                 // weight rows per unit
constexpr int kStages = 4;
constexpr uint32_t kStageBytes = 32768;
constexpr int kConsumers = 4;
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kMaxContrib = 8;
constexpr int kPhases = 3;
constexpr size_t kSmem = kStages * kStageBytes + 1024 + 256;
constexpr int kPlane = kRows * 16;        // one [64 rows][16 x rows] fp32 partial
constexpr size_t kCtaSlotBytes = 2 /*first, last block*/ * 2 /*gate, up*/ * kPlane * 4;
constexpr int kMaxRowBlocks = 4096;       // per phase: up to 262144 weight rows
constexpr int kMaxCtas = 256;

struct Phase {
  const __nv_bfloat16* x;  // [m, k] input rows
  int64_t ldx;
  __nv_bfloat16* y;        // [m, n] output rows
  int64_t ldy;
  const __nv_bfloat16* res;  // residual added in the epilogue (or null)
  int64_t ldres;
  int n, k, nkc, units;
  int gated;
  int map;                 // index of the phase's first tensor map (gated: gate, up)
  unsigned* cnt;           // row-block counters of this phase
};

struct NormTail {          // summed = in + res; normed = rmsnorm(summed) * w
  const __nv_bfloat16* in;
  const __nv_bfloat16* res;
  const void* w;
  int w_dtype;
  float eps;
  __nv_bfloat16* normed;
  __nv_bfloat16* summed;
  int64_t ld;              // leading dimension of all four (rows of n)
  int n;
};

struct ChainArgs {
  Phase ph[kPhases];
  NormTail tail;           // after phase 0
  int m;
  int ctas;
  float* slots;            // [ctas][first, last][gate, up][64][16]
  unsigned* bar;           // [kPhases] barrier counters, zero between launches
  uint32_t* err;
  long long wait_limit;
};

struct ChainMaps {
  CUtensorMap m[4];        // o, gate, up, down
};

__device__ __forceinline__ int unit_begin(int c, int units, int ctas) {
  return static_cast<int>((static_cast<long long>(c) * units) / ctas);
}
__device__ __forceinline__ int cta_of(int u, int units, int ctas) {
  return static_cast<int>(((static_cast<long long>(u) + 1) * ctas + units - 1) / units) - 1;
}

// Bounded spin until *p >= target (gpu-scope acquire). False (after flagging the error
// word and the CTA abort flag) if the limit runs out.
__device__ __forceinline__ bool spin_until(const unsigned* p, unsigned target, uint32_t* err,
                                           volatile int* abort_flag, long long limit) {
  const long long start = clock64();
  for (uint32_t i = 0;; ++i) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    if ((i & 63u) == 63u) {
      if (*abort_flag) return false;
      if (clock64() - start > limit) {
        *abort_flag = 1;
        if (err) atomicOr(err, UMIC_DEVERR_WAIT_TIMEOUT);
        return false;
      }
    }
    __nanosleep(64);
  }
}

// The add + RMSNorm tail on the m rows, by the 128 consumer threads of one CTA.
__device__ void norm_tail(const NormTail& t, int m, float* red) {
  const int tid = threadIdx.x;  // 0..127 (consumer warps)
  const int warp = tid >> 5, lane = tid & 31;
  const int chunks = t.n >> 3;
  for (int r = 0; r < m; ++r) {
    float q = 0.f;
    for (int c = tid; c < chunks; c += kConsumers * 32) {
      float a[8], b[8];
      unpack8(*reinterpret_cast<const uint4*>(t.in + r * t.ld + c * 8), a);
      unpack8(*reinterpret_cast<const uint4*>(t.res + r * t.ld + c * 8), b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        a[j] += b[j];
        q += a[j] * a[j];
      }
      st_vec(t.summed + r * t.ld + c * 8, pack8(a));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    if (lane == 0) red[warp] = q;
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w) tot += red[w];
    const float rstd = rsqrtf(tot / static_cast<float>(t.n) + t.eps);
    // normalise the fp32 sum (recomputed from the inputs, not from the rounded `summed`),
    // as the unfused add+RMSNorm kernel does
    for (int c = tid; c < chunks; c += kConsumers * 32) {
      float a[8], b[8], w8[8];
      unpack8(*reinterpret_cast<const uint4*>(t.in + r * t.ld + c * 8), a);
      unpack8(*reinterpret_cast<const uint4*>(t.res + r * t.ld + c * 8), b);
      load_w8(t.w, t.w_dtype, c * 8, w8);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = (a[j] + b[j]) * rstd * w8[j];
      st_vec(t.normed + r * t.ld + c * 8, pack8(a));
    }
  }
}

template <int MC>
__global__ void __launch_bounds__(kThreads, 1)
    decode_chain_kernel(const __grid_constant__ ChainMaps maps, ChainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  // flags[0]: abort, flags[1]: "this CTA finishes the current row block",
  // flags[2]: "this CTA runs the phase tail"; red: tail reduction scratch
  volatile int* flags = reinterpret_cast<volatile int*>(bars + 2 * kStages);
  float* red = reinterpret_cast<float*>(bars + 2 * kStages) + 8;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStages);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kConsumers);
    }
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < 4; ++i) prefetch_map(&maps.m[i]);
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      for (int p = 0; p < kPhases && ok; ++p) {
        const Phase& ph = a.ph[p];
        const int u0 = unit_begin(c, ph.units, a.ctas), u1 = unit_begin(c + 1, ph.units, a.ctas);
        const int kkc = ph.gated ? 128 : 256;
        for (int u = u0; u < u1; ++u) {
          const int rb = u / ph.nkc, kc = u - rb * ph.nkc;
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, a.err, flags, a.wait_limit)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8 * stage;
          const uint32_t dst = sbase + stage * kStageBytes;
          mbar_expect_tx(fb, kStageBytes);  // out-of-range rows / columns arrive as zeros
          const CUtensorMap* m0 = &maps.m[ph.map];
          if (ph.gated) {
            const CUtensorMap* m1 = &maps.m[ph.map + 1];
            tma_load_2d(dst, m0, fb, kc * kkc, rb * kRows);
            tma_load_2d(dst + 8192, m0, fb, kc * kkc + 64, rb * kRows);
            tma_load_2d(dst + 16384, m1, fb, kc * kkc, rb * kRows);
            tma_load_2d(dst + 24576, m1, fb, kc * kkc + 64, rb * kRows);
          } else {
#pragma unroll
            for (int b = 0; b < 4; ++b)
              tma_load_2d(dst + b * 8192, m0, fb, kc * kkc + b * 64, rb * kRows);
          }
          issued = true;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (ok) {
        for (int s = 0; s < kStages; ++s) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, a.err, flags, a.wait_limit)) break;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      } else if (issued) {
        const long long t0 = clock64();  // copies in flight land before smem goes away
        while (clock64() - t0 < 4000000LL) {
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  int stage = 0;
  uint32_t sphase = 0;

  for (int p = 0; p < kPhases; ++p) {
    const Phase& ph = a.ph[p];
    const bool gated = ph.gated != 0;
    const int u0 = unit_begin(c, ph.units, a.ctas), u1 = unit_begin(c + 1, ph.units, a.ctas);
    float acc[MC][4], acc2[MC][4];
    auto zero_acc = [&]() {
#pragma unroll
      for (int i = 0; i < MC; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] = 0.f;
          acc2[i][j] = 0.f;
        }
    };
    zero_acc();
    auto slot_for = [&](int cta, int rb) {
      const int side = (rb == unit_begin(cta, ph.units, a.ctas) / ph.nkc) ? 0 : 1;
      return a.slots + (static_cast<size_t>(cta) * 2 + side) * 2 * kPlane;
    };
    auto emit = [&](int rb, int rr, int mcol, float v, float v2) {
      const int nrow = rb * kRows + rr;
      if (nrow >= ph.n || mcol >= a.m) return;
      float o = gated ? v / (1.f + __expf(-v)) * v2 : v;
      if (ph.res) o += bf(ph.res[mcol * ph.ldres + nrow]);
      ph.y[mcol * ph.ldy + nrow] = __float2bfloat16_rn(o);
    };
    // Writes row block rb: directly when this CTA holds all of it, else through the slots
    // (the last contributor sums them in CTA order).
    auto flush = [&](int rb) {
      const int first = cta_of(rb * ph.nkc, ph.units, a.ctas);
      const int last = cta_of((rb + 1) * ph.nkc - 1, ph.units, a.ctas);
      const int contrib = last - first + 1;
      if (contrib == 1) {
#pragma unroll
        for (int mc = 0; mc < MC; ++mc)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            emit(rb, j < 2 ? r0 : r1, mc * 8 + 2 * t + (j & 1), acc[mc][j], acc2[mc][j]);
        return;
      }
      float* mine = slot_for(c, rb);
#pragma unroll
      for (int mc = 0; mc < MC; ++mc)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int rr = j < 2 ? r0 : r1, mcol = mc * 8 + 2 * t + (j & 1);
          __stcg(mine + rr * 16 + mcol, acc[mc][j]);
          if (gated) __stcg(mine + kPlane + rr * 16 + mcol, acc2[mc][j]);
        }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
      if (warp == 0 && lane == 0) {
        unsigned prev;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(ph.cnt + rb)
                     : "memory");
        flags[1] = prev == static_cast<unsigned>(contrib - 1);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
      if (!flags[1]) return;
      // partials summed in CTA order (deterministic), straight from L2
#pragma unroll
      for (int mc = 0; mc < MC; ++mc)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int rr = j < 2 ? r0 : r1, mcol = mc * 8 + 2 * t + (j & 1);
          float v = 0.f, v2 = 0.f;
          for (int q = 0; q < contrib; ++q) {
            const float* src = slot_for(first + q, rb);
            v += __ldcg(src + rr * 16 + mcol);
            if (gated) v2 += __ldcg(src + kPlane + rr * 16 + mcol);
          }
          emit(rb, rr, mcol, v, v2);
        }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
      if (warp == 0 && lane == 0) {
        ph.cnt[rb] = 0;  // ready for the next launch
        flags[1] = 0;
      }
    };

    int cur = -1;
    bool ok = true;
    for (int u = u0; u < u1; ++u) {
      const int rb = u / ph.nkc, kc = u - rb * ph.nkc;
      if (rb != cur) {
        if (cur >= 0) {
          flush(cur);
          zero_acc();
        }
        cur = rb;
      }
      const int kkc = gated ? 128 : 256;
      // this unit's activations (written earlier in this kernel or by the previous one:
      // plain coherent loads after the phase barrier's acquire)
      uint4 xv[8][MC];
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const int kk = kc * kkc + s * 32 + t * 8;
#pragma unroll
        for (int mc = 0; mc < MC; ++mc) {
          const int xr = mc * 8 + g;
          const bool live = (gated ? s < 4 : true) && kk < ph.k && xr < a.m;
          xv[s][mc] = live ? *reinterpret_cast<const uint4*>(ph.x + xr * ph.ldx + kk) : zero;
        }
      }
      if (!mbar_wait(full0 + 8 * stage, sphase, a.err, flags, a.wait_limit)) {
        ok = false;
        break;
      }
      const uint32_t st = sbase + stage * kStageBytes;
      if (gated) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint32_t box = st + (s >> 1) * 8192;
          const int chunk = (s & 1) * 4 + t;
          const uint4 wl = lds128(st_swz(box, r0, chunk));
          const uint4 wh = lds128(st_swz(box, r1, chunk));
          const uint4 ul = lds128(st_swz(box + 16384, r0, chunk));
          const uint4 uh = lds128(st_swz(box + 16384, r1, chunk));
#pragma unroll
          for (int mc = 0; mc < MC; ++mc) {
            slab_mma(acc[mc], wl, wh, xv[s][mc]);
            slab_mma(acc2[mc], ul, uh, xv[s][mc]);
          }
        }
      } else {
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t box = st + (s >> 1) * 8192;
          const int chunk = (s & 1) * 4 + t;
          const uint4 wl = lds128(st_swz(box, r0, chunk));
          const uint4 wh = lds128(st_swz(box, r1, chunk));
#pragma unroll
          for (int mc = 0; mc < MC; ++mc) slab_mma(acc[mc], wl, wh, xv[s][mc]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * stage);
      if (++stage == kStages) {
        stage = 0;
        sphase ^= 1;
      }
    }
    if (!ok) return;  // every consumer warp fails the same wait (shared abort flag)
    if (cur >= 0) flush(cur);

    // ---- grid barrier after phase p (and the tail of phase 0)
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    const bool has_tail = p == 0;
    const bool final_phase = p + 1 == kPhases;
    if (warp == 0 && lane == 0) {
      unsigned prev;
      asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                   : "=r"(prev)
                   : "l"(a.bar + p)
                   : "memory");
      flags[2] = prev == static_cast<unsigned>(a.ctas - 1);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    const bool last = flags[2] != 0;
    if (final_phase) {
      if (last && warp == 0 && lane == 0) {
        // every CTA has arrived at the final barrier, so none reads a counter again
        for (int q = 0; q < kPhases; ++q) a.bar[q] = 0;
      }
      return;
    }
    if (has_tail && last) {
      norm_tail(a.tail, a.m, red);
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
      if (warp == 0 && lane == 0)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar + p) : "memory");
    }
    if (warp == 0 && lane == 0) {
      const unsigned target = static_cast<unsigned>(a.ctas) + (has_tail ? 1u : 0u);
      if (!spin_until(a.bar + p, target, a.err, flags, a.wait_limit)) flags[0] = 1;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    if (flags[0]) return;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
}

// ------------------------------------------------------------------- host

size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

size_t counters_offset(int ctas) { return align256(static_cast<size_t>(ctas) * kCtaSlotBytes); }

size_t workspace_bytes() {
  return counters_offset(kMaxCtas) + align256(kPhases * kMaxRowBlocks * 4) + 256;
}

template <int MC>
int launch(const ChainMaps& maps, const ChainArgs& a, cudaStream_t st) {
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    e = cudaFuncSetAttribute(decode_chain_kernel<MC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmem));
  });
  if (e != cudaSuccess)
    return fail(UMIC_ERR_LAUNCH, "umic_decode_mlp_chain: smem attribute: %s",
                cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, decode_chain_kernel<MC>, maps, a);
  if (e != cudaSuccess)
    return fail(UMIC_ERR_LAUNCH, "umic_decode_mlp_chain: %s", cudaGetErrorString(e));
  return launch_status("umic_decode_mlp_chain");
}

bool aligned_ld(int64_t ld) { return ld > 0 && ld % 8 == 0; }

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" {

size_t umic_decode_chain_workspace_bytes(void) { return workspace_bytes(); }

int umic_decode_mlp_chain(const void* attn, int64_t ld_attn, const void* w_o, int64_t ld_wo,
                          const void* residual, int64_t ld_res, const void* post_w,
                          int post_w_dtype, float post_eps, const void* w_gate,
                          const void* w_up, int64_t ld_wgu, const void* w_down, int64_t ld_wd,
                          void* out, int64_t ld_out, void* scratch, size_t scratch_bytes,
                          int64_t m, int64_t hidden, int64_t k_attn, int64_t inter,
                          void* workspace, size_t workspace_bytes_, void* stream) {
  static const char* kName = "umic_decode_mlp_chain";
  clear_error();
  if (m < 0 || hidden <= 0 || k_attn <= 0 || inter <= 0)
    return fail(UMIC_ERR_INVALID_ARG, "%s: bad sizes", kName);
  if (m == 0) return UMIC_OK;
  if (m > 16) return fail(UMIC_ERR_UNSUPPORTED, "%s: m=%lld > 16 rows", kName, (long long)m);
  if (!attn || !w_o || !residual || !post_w || !w_gate || !w_up || !w_down || !out ||
      !scratch || !workspace)
    return fail(UMIC_ERR_INVALID_ARG, "%s: null pointer", kName);
  if (post_w_dtype != UMIC_DTYPE_BF16 && post_w_dtype != UMIC_DTYPE_FP32)
    return fail(UMIC_ERR_INVALID_ARG, "%s: bad post_w_dtype", kName);
  if (hidden % 64 || inter % 64 || k_attn % 8)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: hidden and inter must be multiples of 64, the "
                "attention width of 8", kName);
  if (hidden / 64 > kMaxRowBlocks || inter / 64 > kMaxRowBlocks)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: more than %d row blocks", kName, kMaxRowBlocks);
  const void* ptrs[] = {attn, w_o, residual, w_gate, w_up, w_down, out, scratch};
  for (const void* p : ptrs)
    if (!aligned16(p)) return fail(UMIC_ERR_ALIGNMENT, "%s: 16-byte aligned pointers", kName);
  if (!aligned_ld(ld_attn) || !aligned_ld(ld_wo) || !aligned_ld(ld_res) || !aligned_ld(ld_wgu) ||
      !aligned_ld(ld_wd) || !aligned_ld(ld_out) || ld_attn < k_attn || ld_wo < k_attn ||
      ld_res < hidden || ld_wgu < hidden || ld_wd < inter || ld_out < hidden)
    return fail(UMIC_ERR_ALIGNMENT, "%s: leading dimensions must be multiples of 8 covering "
                "the rows", kName);
  // scratch: o, normed, summed [m, hidden] and h [m, inter], each 256-byte aligned
  const size_t row_h = align256(static_cast<size_t>(m) * hidden * 2);
  const size_t need = 3 * row_h + align256(static_cast<size_t>(m) * inter * 2);
  if (scratch_bytes < need)
    return fail(UMIC_ERR_INVALID_ARG, "%s: scratch of %zu bytes, %zu needed", kName,
                scratch_bytes, need);
  if (workspace_bytes_ < workspace_bytes() || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(UMIC_ERR_INVALID_ARG, "%s: workspace must be 256-byte aligned and hold %zu "
                "bytes", kName, workspace_bytes());
  const int ctas = sm_count() < kMaxCtas ? sm_count() : kMaxCtas;
  // every row block within kMaxContrib contributors: at least ceil(nkc / 7) units per CTA
  auto fits = [&](int64_t rows, int64_t k, int kkc) {
    const int64_t nkc = (k + kkc - 1) / kkc, units = (rows / 64) * nkc;
    return units / ctas >= (nkc + kMaxContrib - 2) / (kMaxContrib - 1);
  };
  if (!fits(hidden, k_attn, 256) || !fits(inter, hidden, 128) || !fits(hidden, inter, 256))
    return fail(UMIC_ERR_UNSUPPORTED, "%s: matrices too small to split over %d CTAs", kName,
                ctas);

  ChainMaps maps;
  if (!make_map(&maps.m[0], w_o, hidden, k_attn, ld_wo, 64) ||
      !make_map(&maps.m[1], w_gate, inter, hidden, ld_wgu, 64) ||
      !make_map(&maps.m[2], w_up, inter, hidden, ld_wgu, 64) ||
      !make_map(&maps.m[3], w_down, hidden, inter, ld_wd, 64))
    return fail(UMIC_ERR_DEVICE, "%s: cuTensorMapEncodeTiled unavailable or rejected", kName);

  uint8_t* sc = static_cast<uint8_t*>(scratch);
  auto* o_buf = reinterpret_cast<__nv_bfloat16*>(sc);
  auto* normed = reinterpret_cast<__nv_bfloat16*>(sc + row_h);
  auto* summed = reinterpret_cast<__nv_bfloat16*>(sc + 2 * row_h);
  auto* h_buf = reinterpret_cast<__nv_bfloat16*>(sc + 3 * row_h);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto* cnt = reinterpret_cast<unsigned*>(ws + counters_offset(kMaxCtas));
  auto* bar = cnt + kPhases * kMaxRowBlocks;

  ChainArgs a{};
  auto set = [&](int p, const void* x, int64_t ldx, __nv_bfloat16* y, int64_t ldy,
                 const void* res, int64_t ldres, int64_t n, int64_t k, int gated, int map) {
    Phase& ph = a.ph[p];
    ph.x = static_cast<const __nv_bfloat16*>(x);
    ph.ldx = ldx;
    ph.y = y;
    ph.ldy = ldy;
    ph.res = static_cast<const __nv_bfloat16*>(res);
    ph.ldres = ldres;
    ph.n = static_cast<int>(n);
    ph.k = static_cast<int>(k);
    const int kkc = gated ? 128 : 256;
    ph.nkc = static_cast<int>((k + kkc - 1) / kkc);
    ph.units = static_cast<int>(n / 64) * ph.nkc;
    ph.gated = gated;
    ph.map = map;
    ph.cnt = cnt + p * kMaxRowBlocks;
  };
  set(0, attn, ld_attn, o_buf, hidden, nullptr, 0, hidden, k_attn, 0, 0);
  set(1, normed, hidden, h_buf, inter, nullptr, 0, inter, hidden, 1, 1);
  set(2, h_buf, inter, static_cast<__nv_bfloat16*>(out), ld_out, summed, hidden, hidden, inter, 0,
      3);
  a.tail.in = o_buf;
  a.tail.res = static_cast<const __nv_bfloat16*>(residual);
  a.tail.w = post_w;
  a.tail.w_dtype = post_w_dtype;
  a.tail.eps = post_eps;
  a.tail.normed = normed;
  a.tail.summed = summed;
  a.tail.ld = hidden;
  a.tail.n = static_cast<int>(hidden);
  a.m = static_cast<int>(m);
  a.ctas = ctas;
  a.slots = reinterpret_cast<float*>(ws);
  a.bar = bar;
  a.err = device_error_word();
  a.wait_limit = kWaitLimitCycles;
  if (ld_res != hidden) {
    // the tail reads the residual with the rows' leading dimension: stage it only when
    // it is dense (the decoder's stream always is)
    return fail(UMIC_ERR_UNSUPPORTED, "%s: residual rows must be dense (ld == hidden)", kName);
  }
  cudaStream_t st = as_stream(stream);
  return m <= 8 ? launch<1>(maps, a, st) : launch<2>(maps, a, st);
}

}  // extern "C"
