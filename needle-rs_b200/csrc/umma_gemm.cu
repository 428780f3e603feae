// Codebook-quantized projection on the 5th-generation tensor cores (tcgen05).
//
// y[m][o] = sum_g norm[o,g] * sum_{k in g} level[idx[o,k]] * xh[m,k]   (cq.rs:632-679)
//
// for many activation rows. The tensor cores multiply f16 operands into f32
// accumulators held in tensor memory (TMEM). To keep f32 accuracy both
// operands are split into an f16 high part and an f16 remainder,
// x = x_hi + x_lo and level = l_hi + l_lo, and per 128-element group the
// products x_hi*l_hi, x_lo*l_hi (and x_hi*l_lo) accumulate in one TMEM
// accumulator (f16 products are exact; the dropped x_lo*l_lo term and the
// remainders' rounding leave ~2^-22 per product). The tensor cores' f32
// accumulation truncates toward zero, so an accumulator only ever spans one
// group: after each group the epilogue warps read it and add norm * group dot
// into f32 registers with round-to-nearest, the reference's own
// norm-times-group-dot structure. Every 128-wide group of an activation row
// and the level table are scaled by powers of two that keep each f16
// remainder in the normal range; the epilogue undoes them exactly (the
// activation scale per row and group, the level scale folded into the norms).
// When every scaled level is itself an f16 value (codebooks stored as f16
// numbers, as the packer writes them), the level remainders are zero: that
// form skips their tile and their MMA, two MMAs per K step instead of three.
//
// Operands: the engine's matrices have their level tiles expanded once at
// load (umma_cache_levels); other callers get them from the packed codes per
// call. The split activations come from the kernel that produced the rows
// (the engine's row and attention kernels write this form directly) or from
// a preparation launch (umma_prep_kernel), which also expands uncached levels.
//
// Persistent: one CTA per SM walks tiles of 128 activation rows x UN (64, 128
// or 192) weight rows with UN / 16 + 2 warps:
//   * one warp loads [128 rows x 64 k] tiles of the split activations and of
//     the levels with TMA and 128-byte swizzle into a ring of stages, and owns
//     the TMEM allocation;
//   * one thread issues tcgen05.mma kind::f16 M=128 N=UN K=16, two (three)
//     per K step; the groups of every tile alternate between two accumulators
//     so one is drained while the other fills;
//   * UN / 16 epilogue warps drain the accumulators (warp w reads TMEM lanes
//     32*(w%4).. and 64 columns from 64*(w/4)) and store y through a per-warp
//     shared-memory transpose.
// Every wait on an mbarrier is bounded in time; on expiry the CTA raises a
// device error flag, stops, waits (bounded) for its issued copies and MMAs,
// frees its TMEM and returns, and the host reports the flag.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "kernels.hpp"
#include "launch_util.hpp"

namespace nb {

// Raised when a bounded wait of the tensor-core GEMM gave up and no caller
// flag was given (the standalone nd_cq_project); an engine passes its own.
__device__ int g_umma_error;

namespace {

constexpr int UM = 128;  // activation rows per tile (MMA M)
constexpr int UK = 64;   // K per stage: 64 f16 = one 128-byte swizzle row
// Pipeline of one tile width UN (weight rows per tile, the MMA N: 64, 128 or 192).
// A stage holds the activation tiles (high part and remainder, [128 rows][64 k]
// f16 each) and the level tile(s) ([UN rows][64 k] f16; remainders too unless
// the levels are exact), in as many stages as fit 192 KB.
template <bool EXACT, int UN>
struct Pipe {
  static constexpr uint32_t A_TILE = UM * 128;
  static constexpr uint32_t B_TILE = UN * 128;
  static constexpr uint32_t STAGE_BYTES = 2 * A_TILE + (EXACT ? 1u : 2u) * B_TILE;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int EPI_WARPS = UN / 16;             // lane quarter x 64-column block
  static constexpr int THREADS = (EPI_WARPS + 2) * 32;  // + TMA / TMEM warp + MMA warp
};
constexpr int UGMAX = 32;  // groups of 128 supported (in_pad <= 4096)
// Output staging of one epilogue warp: 32 rows x 16 columns, rows 20 floats
// apart (float4 writes of a row per lane and float4 reads of 8 rows x 64
// bytes per warp instruction are both bank-conflict free or nearly).
constexpr int OST = 20;
constexpr uint32_t OUT_STAGE = 32 * OST * 4;
// Dynamic shared memory: alignment slack, the stages, the norm table of one
// tile ([groups][UN] f32), the barriers and (when it fits: every shipped
// shape) the epilogue warps' output staging.
template <bool EXACT, int UN>
constexpr size_t umma_smem(int groups, bool out_stage) {
  return 1024 + (size_t)Pipe<EXACT, UN>::STAGES * Pipe<EXACT, UN>::STAGE_BYTES + (size_t)groups * UN * 4 + 256 +
         (out_stage ? (size_t)Pipe<EXACT, UN>::EPI_WARPS * OUT_STAGE : 0);
}
constexpr unsigned long long WAIT_NS = 1000000000ull;  // bound of every wait: one second

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(su32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar`. Gives up after WAIT_NS (raising *werr) or
// as soon as another role of the CTA gave up (`abort`), returning false. Between polls a
// waiter sleeps `backoff_ns` so waiting warps leave the issue slots to the
// warps that decode weights on the same schedulers.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort, int* werr,
                                          unsigned backoff_ns = 0) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = now_ns();
  while (true) {
    if (backoff_ns) __nanosleep(backoff_ns);
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (now_ns() - t0 > WAIT_NS) {
      *abort = 1;
      atomicExch(werr, 1);
      return false;
    }
  }
}

// Drain wait used on the abort path: ignores the abort flag, bounded in time.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = now_ns();
  while (!mbar_try(bar, parity) && now_ns() - t0 <= WAIT_NS) {
  }
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(su32(bar)), "r"(x), "r"(y)
      : "memory");
}

// K-major operand tile, 128-byte swizzle: rows of 128 B, 8-row atoms 1024 B
// apart (stride byte offset), start address in 16-byte units.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t start = (su32(tile) & 0x3FFFF) >> 4;
  return start | (uint64_t)(1024 >> 4) << 32 | (uint64_t)1 << 46 | (uint64_t)2 << 61;
}

// kind::f16 instruction descriptor: f32 accumulate, f16 A and B, both K-major,
// M = 128, N = UN.
template <int UN>
constexpr uint32_t idesc() {
  return (1u << 4) | ((uint32_t)(UN >> 3) << 17) | ((uint32_t)(UM >> 4) << 24);
}

template <int UN>
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc<UN>()), "r"(accum));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// EXACT: every level times the level scale is an f16 value, so the level
// remainders are zero and only x_hi * l_hi and x_lo * l_hi are issued (two
// MMAs per K step, no remainder tile).
//
// Persistent: CTA b computes tiles b, b + gridDim.x, ... of 128 activation
// rows x UN weight rows (tile t: activation rows (t / ntn) * 128, weight rows
// (t % ntn) * UN, so CTAs running at the same time share activation tiles in
// L2). Every MMA of a quantisation group accumulates into one TMEM accumulator
// of UN columns; the groups of every tile alternate between two accumulators,
// so the epilogue drains one (its last group of a tile included) while the
// MMAs of the next group, of this tile or the next, fill the other.
template <bool EXACT, int UN>
__global__ void __launch_bounds__(Pipe<EXACT, UN>::THREADS, 1)
cq_umma_kernel(CqMat W, const __grid_constant__ CUtensorMap mapAh, const __grid_constant__ CUtensorMap mapAl,
               const __grid_constant__ CUtensorMap mapBh, const __grid_constant__ CUtensorMap mapBl,
               const float* __restrict__ ainv, float linv, int M, float* __restrict__ y, int ldy, int row0,
               int nrows, int ntn, int ntiles, int* werr, int out_stage, unsigned long long* __restrict__ amax) {
  pdl_trigger();  // the consumer of y may launch now; it waits for this grid before reading y
  using P = Pipe<EXACT, UN>;
  constexpr int USTAGES = P::STAGES;
  constexpr uint32_t STAGE_BYTES = P::STAGE_BYTES;
  constexpr int EW = P::EPI_WARPS;
  constexpr uint32_t TMEM_COLS = 2 * UN <= 128 ? 128 : 2 * UN <= 256 ? 256 : 512;  // two group accumulators
  extern __shared__ unsigned char smraw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  const int nk = W.in_pad / UK, ng = W.in_pad / 128;
  float* nsm = reinterpret_cast<float*>(sm + USTAGES * STAGE_BYTES);  // [ng][UN]
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + USTAGES * STAGE_BYTES + (size_t)ng * UN * 4);
  uint64_t* empty = full + USTAGES;   // stage consumed by the MMAs
  uint64_t* tfull = empty + USTAGES;  // [2] a group's accumulator is complete
  uint64_t* tempty = tfull + 2;       // [2] the accumulator has been drained
  uint64_t* drainb = tempty + 2;      // every MMA of the CTA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drainb + 1);
  volatile uint32_t* abort = tmem_slot + 1;
  float* ostage = reinterpret_cast<float*>(sm + USTAGES * STAGE_BYTES + (size_t)ng * UN * 4 + 256);  // [EW][32][OST]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < USTAGES; ++s) {
      mbar_init(&full[s], 1);   // the TMA thread's expect_tx arrive
      mbar_init(&empty[s], 1);  // one tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);    // one tcgen05.commit
      mbar_init(&tempty[b], EW);  // the epilogue warps
    }
    mbar_init(drainb, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == EW) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launched with programmatic dependent launch: the set-up above overlaps the
  // producer of the activations; everything below reads what it wrote.
  pdl_wait();

  if (warp < EW) {
    // ------------------------------------------------ epilogue: drain each group
    // Warp w reads TMEM lanes 32 * (w % 4).. (its lane quarter) and columns
    // 64 * (w / 4).. of each accumulator.
    const int q = warp & 3, cq = warp >> 2;
    bool ok = true;
    int gg = 0;  // groups drained so far, over every tile of this CTA
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const int m0 = (t / ntn) * UM, n0 = (t % ntn) * UN;
      // Group norms of the tile's weight rows times the inverse level scale,
      // rebuilt once every epilogue warp is done with the previous tile's.
      asm volatile("bar.sync 1, %0;" ::"r"(EW * 32) : "memory");
      for (int nl = tid; nl < UN; nl += EW * 32) {
        const __half* pn = nullptr;
        if (n0 + nl < nrows) {
          const uint8_t* prow;
          cq_row_ptr(W, row0 + n0 + nl, &prow, &pn);
        }
        for (int g = 0; g < ng; ++g) nsm[g * UN + nl] = pn ? __half2float(pn[g]) * linv : 0.f;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(EW * 32) : "memory");
      float acc[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0.f;
      const int m = m0 + q * 32 + lane;
      const float* arow = ainv + (size_t)(m < M ? m : 0) * ng;  // this row's group scales
      for (int g = 0; g < ng; ++g, ++gg) {
        const int b = gg & 1;
        const float ag = arow[g];  // in flight while the group completes
        if (ok && !mbar_wait(&tfull[b], (uint32_t)(gg >> 1) & 1u, abort, werr, 128)) ok = false;
        if (!ok) continue;
        tc_fence_after();
        const uint32_t tm = tmem + ((uint32_t)(q * 32) << 16) + b * UN + cq * 64;
        const float* ngp = nsm + g * UN + cq * 64;
        // Two TMEM loads per wait where the registers allow (the 14-warp
        // UN = 192 CTA is held to 128 registers a thread).
        constexpr int LPW = UN >= 192 ? 1 : 2;
#pragma unroll
        for (int cb = 0; cb < 4; cb += LPW) {
          uint32_t r[LPW][16];
#pragma unroll
          for (int h = 0; h < LPW; ++h) tmem_ld16(tm + (cb + h) * 16, r[h]);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < LPW; ++h)
#pragma unroll
            for (int i = 0; i < 16; ++i)
              acc[(cb + h) * 16 + i] += (ngp[(cb + h) * 16 + i] * ag) * __uint_as_float(r[h][i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
      const int lim = nrows - (n0 + cq * 64);
      // Warp-uniform: the warp's 32 rows x 64 columns lie inside y and every
      // row start is 16-byte aligned. The rows then leave through shared
      // memory, 16 columns at a time, so that one store instruction writes 8
      // rows x 64 contiguous bytes instead of 32 rows x 16 bytes.
      const bool vec = out_stage && ok && m0 + q * 32 + 32 <= M && lim >= 64 && (ldy & 3) == 0 &&
                       (reinterpret_cast<uintptr_t>(y + n0 + cq * 64) & 15) == 0;
      if (amax) {  // greedy pick: the row's best key over this warp's columns
        if (ok && m < M) {
          unsigned long long best = 0ull;
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i < lim && acc[i] == acc[i]) best = max(best, argmax_key(acc[i], (uint32_t)(n0 + cq * 64 + i)));
          if (best) atomicMax(amax + m, best);
        }
      } else if (vec) {
        float* ob = ostage + (size_t)warp * 32 * OST;
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(ob + lane * OST + i) =
                make_float4(acc[cb * 16 + i], acc[cb * 16 + i + 1], acc[cb * 16 + i + 2], acc[cb * 16 + i + 3]);
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int rr = it * 8 + (lane >> 2), c4 = (lane & 3) * 4;
            *reinterpret_cast<float4*>(y + (size_t)(m0 + q * 32 + rr) * ldy + n0 + cq * 64 + cb * 16 + c4) =
                *reinterpret_cast<const float4*>(ob + rr * OST + c4);
          }
          __syncwarp();
        }
      } else if (ok && m < M) {
        float* yr = y + (size_t)m * ldy + n0 + cq * 64;
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < lim) yr[i] = acc[i];
      }
    }
  } else if (warp == EW) {
    // ------------------------------------------------ operand producer (TMA)
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        const int m0 = (t / ntn) * UM, n0 = (t % ntn) * UN;
        for (int kb = 0; kb < nk; ++kb) {
          const int s = issued % USTAGES;
          const uint32_t ph = (uint32_t)(issued / USTAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abort, werr)) {
            ok = false;
            break;
          }
          unsigned char* st = sm + s * STAGE_BYTES;
          mbar_arrive_tx(&full[s], STAGE_BYTES);
          tma_load_2d(st, &mapAh, &full[s], kb * UK, m0);
          tma_load_2d(st + P::A_TILE, &mapAl, &full[s], kb * UK, m0);
          tma_load_2d(st + 2 * P::A_TILE, &mapBh, &full[s], kb * UK, n0);
          if (!EXACT) tma_load_2d(st + 2 * P::A_TILE + P::B_TILE, &mapBl, &full[s], kb * UK, n0);
          ++issued;
        }
      }
      if (*abort) {  // let the copies already issued land before the CTA exits
        for (int kb = issued - USTAGES > 0 ? issued - USTAGES : 0; kb < issued; ++kb)
          mbar_drain(&full[kb % USTAGES], (uint32_t)(kb / USTAGES) & 1u);
      }
    }
  } else {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int kb = 0, gg = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        for (int g = 0; g < ng && ok; ++g, ++gg) {
          const int b = gg & 1;
          if (!mbar_wait(&tempty[b], ((uint32_t)(gg >> 1) & 1u) ^ 1u, abort, werr)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + b * UN;
          for (int j = 0; j < 2; ++j, ++kb) {
            const int s = kb % USTAGES;
            const uint32_t ph = (uint32_t)(kb / USTAGES) & 1u;
            if (!mbar_wait(&full[s], ph, abort, werr)) {
              ok = false;
              break;
            }
            tc_fence_after();
            unsigned char* st = sm + s * STAGE_BYTES;
            const uint64_t dah = sw128_desc(st), dal = sw128_desc(st + P::A_TILE);
            const uint64_t dbh = sw128_desc(st + 2 * P::A_TILE), dbl = sw128_desc(st + 2 * P::A_TILE + P::B_TILE);
#pragma unroll
            for (int kk = 0; kk < UK / 16; ++kk) {
              const uint64_t o = (uint64_t)(kk * 2);  // 32 bytes along K, in 16-byte units
              umma_f16<UN>(d, dah + o, dbh + o, (j | kk) != 0);  // a group starts from zero
              umma_f16<UN>(d, dal + o, dbh + o, 1);
              if (!EXACT) umma_f16<UN>(d, dah + o, dbl + o, 1);
            }
            umma_commit(&empty[s]);
          }
          if (ok) umma_commit(&tfull[b]);
        }
      }
      // Every issued MMA completes before TMEM is freed.
      umma_commit(drainb);
      mbar_drain(drainb, 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == EW) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// Level high parts and remainders of rows [row0, row0 + nrows) of a CQ
// matrix, decoded from the packed codes (cq.rs:908-925) and scaled by 2^le:
// hi / lo [nrows][in_pad] f16 (no remainders when wlo is null: exact levels).
// One thread per 8 weights; block `blk` of `nblk` strides over the rows.
template <int BITS>
__device__ __forceinline__ void expand_levels(const CqMat& W, int row0, int nrows, int le, __half* __restrict__ whi,
                                              __half* __restrict__ wlo, int blk, int nblk) {
  __shared__ uint32_t tab[16];  // level * 2^le as (hi | lo << 16)
  if (threadIdx.x < 16) tab[threadIdx.x] = split_h16(ldexpf(W.levels[threadIdx.x < (1 << BITS) ? threadIdx.x : 0], le));
  __syncthreads();
  const int per_row = W.in_pad / 8;
  const long total = (long)nrows * per_row;
  for (long i = blk * (long)blockDim.x + threadIdx.x; i < total; i += (long)nblk * blockDim.x) {
    const int n = (int)(i / per_row), c = (int)(i % per_row);
    const uint8_t* prow;
    const __half* pn;
    cq_row_ptr(W, row0 + n, &prow, &pn);
    uint32_t code = BITS == 2 ? (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(prow) + c)
                              : __ldg(reinterpret_cast<const uint32_t*>(prow) + c);
    uint32_t h[4], l[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t a = tab[(code >> (2 * p * BITS)) & ((1u << BITS) - 1)];
      const uint32_t b = tab[(code >> ((2 * p + 1) * BITS)) & ((1u << BITS) - 1)];
      h[p] = __byte_perm(a, b, 0x5410);
      l[p] = __byte_perm(a, b, 0x7632);
    }
    *reinterpret_cast<uint4*>(whi + (size_t)n * W.in_pad + c * 8) = make_uint4(h[0], h[1], h[2], h[3]);
    if (wlo) *reinterpret_cast<uint4*>(wlo + (size_t)n * W.in_pad + c * 8) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// f32 activations [M][ldx] -> row-scaled f16 high parts and remainders
// [M][K] and the inverse row scales [M]. One warp per row (block `blk`: rows
// blk * 8 ..).
// Activation rows [M][K] f32 -> hi / lo [M][K] f16 and inv [M][K / 128], each
// 128-wide group scaled on its own (split_group_store); one warp per row.
__device__ __forceinline__ void split_rows(const float* __restrict__ x, int ldx, int M, int K, __half* __restrict__ hi,
                                           __half* __restrict__ lo, float* __restrict__ inv, int blk) {
  const int lane = threadIdx.x & 31;
  const int m = blk * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (m >= M) return;  // the whole warp
  const float* xr = x + (size_t)m * ldx;
  const int ng = K / 128;
  for (int g = 0; g < ng; ++g) {
    const float4 a = *reinterpret_cast<const float4*>(xr + g * 128 + lane * 4);
    const float v[4] = {a.x, a.y, a.z, a.w};
    split_group_store(v, hi + (size_t)m * K + g * 128, lo + (size_t)m * K + g * 128, inv + (size_t)m * ng + g);
  }
}

// Both operand preparations of one projection in one launch (they are
// independent): blocks below `split_blocks` split activation rows (split_f16),
// the others expand level tiles (cq_expand).
template <int BITS>
__global__ void __launch_bounds__(256) umma_prep_kernel(const float* __restrict__ x, int ldx, int M, int K,
                                                        __half* __restrict__ hi, __half* __restrict__ lo,
                                                        float* __restrict__ inv, int split_blocks, CqMat W, int row0,
                                                        int nrows, int le, __half* __restrict__ whi,
                                                        __half* __restrict__ wlo) {
  if ((int)blockIdx.x < split_blocks) {
    split_rows(x, ldx, M, K, hi, lo, inv, blockIdx.x);
    return;
  }
  expand_levels<BITS>(W, row0, nrows, le, whi, wlo, blockIdx.x - split_blocks, gridDim.x - split_blocks);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor map of an f16 [M][K] row-major array: box [box_rows rows][64 k], 128-byte swizzle.
bool make_map(CUtensorMap* map, const __half* base, int M, int K, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)UK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// whi / wlo: the level tiles of rows [row0, row0 + nrows) ([nrows][in_pad] f16).
template <bool EXACT, int UN>
cudaError_t launch_umma(const CqMat& W, const GemmScratch& gs, const __half* whi, const __half* wlo, float linv,
                        int M, float* y, int ldy, int row0, int nrows, int* werr, cudaStream_t st) {
  const int K = W.in_pad;
  CUtensorMap mah, mal, mbh, mbl;
  if (!make_map(&mah, gs.hi, M, K, UM) || !make_map(&mal, gs.lo, M, K, UM) || !make_map(&mbh, whi, nrows, K, UN) ||
      !make_map(&mbl, wlo, nrows, K, UN))
    return cudaErrorNotSupported;
  auto kern = cq_umma_kernel<EXACT, UN>;
  const bool out_stage = umma_smem<EXACT, UN>(K / 128, true) <= 227 * 1024;
  const size_t smem = umma_smem<EXACT, UN>(K / 128, out_stage);
  cudaError_t e = allow_smem((const void*)kern, smem);
  if (e != cudaSuccess) return e;
  const int ntn = (nrows + UN - 1) / UN, ntiles = ntn * ((M + UM - 1) / UM);
  const int grid = std::min(ntiles, 148);  // persistent: one CTA per SM
  return launch_pdl(kern, dim3(grid), dim3(Pipe<EXACT, UN>::THREADS), smem, st, W, mah, mal, mbh, mbl, gs.inv, linv,
                    M, y, ldy, row0, nrows, ntn, ntiles, werr, out_stage ? 1 : 0, gs.amax);
}

}  // namespace

bool umma_supported(const CqMat& W) {
  return W.group == 128 && (W.bits == 2 || W.bits == 4) && W.in_pad % 128 == 0 && W.in_pad <= UGMAX * 128;
}

// Level scale of the f16 level tiles: a power of two 2^le putting max|level|
// in [2^13, 2^14); exact when every scaled level survives the round trip
// through f16 (then the tiles need no remainders).
static void umma_level_scale(const CqMat& W, int* le_out, bool* exact_out) {
  float lmax = 0.f;
  for (int i = 0; i < (1 << W.bits); ++i) lmax = std::max(lmax, std::fabs(W.levels[i]));
  int le = 0;
  if (lmax > 0.f && std::isfinite(lmax)) {
    int e;
    std::frexp(lmax, &e);
    le = 14 - e;
  }
  bool exact = true;
  for (int i = 0; i < (1 << W.bits); ++i) {
    const float v = std::ldexp(W.levels[i], le);
    if (__half2float(__float2half_rn(v)) != v) exact = false;
  }
  *le_out = le;
  *exact_out = exact;
}

template <int BITS>
__global__ void __launch_bounds__(256) expand_all_kernel(CqMat W, int le, __half* __restrict__ whi,
                                                         __half* __restrict__ wlo) {
  expand_levels<BITS>(W, 0, W.rows, le, whi, wlo, blockIdx.x, gridDim.x);
}

cudaError_t umma_cache_levels(CqMat* W, std::vector<void*>* owned, cudaStream_t st) {
  if (!umma_supported(*W) || W->lvl_hi) return cudaSuccess;
  int le;
  bool exact;
  umma_level_scale(*W, &le, &exact);
  const size_t n = (size_t)W->rows * W->in_pad;
  __half *hi = nullptr, *lo = nullptr;
  cudaError_t e = cudaMalloc(&hi, n * sizeof(__half));
  if (e == cudaSuccess && !exact) e = cudaMalloc(&lo, n * sizeof(__half));
  if (e == cudaSuccess) {
    const long total = (long)W->rows * (W->in_pad / 8);
    const int blocks = (int)std::min<long>((total + 255) / 256, 148L * 8);
    if (W->bits == 2)
      expand_all_kernel<2><<<blocks, 256, 0, st>>>(*W, le, hi, lo);
    else
      expand_all_kernel<4><<<blocks, 256, 0, st>>>(*W, le, hi, lo);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    if (hi) cudaFree(hi);
    if (lo) cudaFree(lo);
    return e;
  }
  owned->push_back(hi);
  if (lo) owned->push_back(lo);
  W->lvl_hi = hi;
  W->lvl_lo = lo;
  return cudaSuccess;
}

cudaError_t cq_project_umma(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy, int row0,
                            int nrows, cudaStream_t st, const GemmScratch& gs, bool presplit) {
  const int K = W.in_pad;
  if (!umma_supported(W) || !gs.hi || !gs.lo || !gs.inv || !gs.whi || !gs.wlo || gs.elems < (size_t)M * K ||
      gs.rows < (size_t)M || gs.welems < (size_t)nrows * K)
    return cudaErrorInvalidValue;
  const uintptr_t al = reinterpret_cast<uintptr_t>(gs.hi) | reinterpret_cast<uintptr_t>(gs.lo) |
                       reinterpret_cast<uintptr_t>(gs.whi) | reinterpret_cast<uintptr_t>(gs.wlo);
  if (al & 15) return cudaErrorInvalidValue;
  int le;
  bool exact;
  umma_level_scale(W, &le, &exact);
  // Level tiles expanded at load (the engine's matrices) or now, into scratch.
  const bool cached = W.lvl_hi && (exact || W.lvl_lo);
  const __half* whi = cached ? W.lvl_hi + (size_t)row0 * K : gs.whi;
  const __half* wlo = cached ? (W.lvl_lo ? W.lvl_lo + (size_t)row0 * K : whi) : gs.wlo;
  cudaError_t e;
  {
    // presplit: the producer of xh already wrote gs.hi / lo / inv.
    const int split_blocks = presplit ? 0 : (M + 7) / 8;
    const long total = (long)nrows * (K / 8);
    const int eblocks = cached ? 0 : (int)std::min<long>((total + 255) / 256, 148L * 8);
    __half* xwlo = exact ? nullptr : gs.wlo;  // remainders, when the levels need them
    if (split_blocks + eblocks > 0) {  // else nothing to prepare: the projection is one launch
      if (W.bits == 2)
        umma_prep_kernel<2><<<split_blocks + eblocks, 256, 0, st>>>(xh, ldx, M, K, gs.hi, gs.lo, gs.inv,
                                                                    split_blocks, W, row0, nrows, le, gs.whi, xwlo);
      else
        umma_prep_kernel<4><<<split_blocks + eblocks, 256, 0, st>>>(xh, ldx, M, K, gs.hi, gs.lo, gs.inv,
                                                                    split_blocks, W, row0, nrows, le, gs.whi, xwlo);
      e = cudaGetLastError();
      if (e != cudaSuccess) return e;
    }
  }
  int* werr = gs.werr;
  if (!werr) {
    e = umma_error_ptr(&werr);
    if (e != cudaSuccess) return e;
  }
  // Tile width by makespan: rounds of tiles over the 148 SMs times a tile's
  // operand bytes (128 activation rows x 4 B + UN weight rows x 2 B per K;
  // the operands stream from L2), the wider tile on a tie. 64-row tiles put
  // more SMs to work on small batches; 192 keeps the 14-warp CTA at 128
  // registers a thread (256 would spill).
  const float linv = std::ldexp(1.f, -le);
  const long mt = (M + UM - 1) / UM;
  auto span = [&](long un) { return (((nrows + un - 1) / un) * mt + 147) / 148 * (512 + 2 * un); };
  const int un = span(192) <= span(128) ? 192 : span(128) <= span(64) ? 128 : 64;
  if (exact)
    return un == 192   ? launch_umma<true, 192>(W, gs, whi, wlo, linv, M, y, ldy, row0, nrows, werr, st)
           : un == 128 ? launch_umma<true, 128>(W, gs, whi, wlo, linv, M, y, ldy, row0, nrows, werr, st)
                       : launch_umma<true, 64>(W, gs, whi, wlo, linv, M, y, ldy, row0, nrows, werr, st);
  return un == 192   ? launch_umma<false, 192>(W, gs, whi, wlo, linv, M, y, ldy, row0, nrows, werr, st)
         : un == 128 ? launch_umma<false, 128>(W, gs, whi, wlo, linv, M, y, ldy, row0, nrows, werr, st)
                     : launch_umma<false, 64>(W, gs, whi, wlo, linv, M, y, ldy, row0, nrows, werr, st);
}

cudaError_t umma_error_ptr(int** p) { return cudaGetSymbolAddress((void**)p, g_umma_error); }

cudaError_t umma_take_error(int* flag) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_umma_error, sizeof(int));
  if (e == cudaSuccess && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_umma_error, &zero, sizeof(int));
  }
  *flag = v;
  return e;
}

}  // namespace nb
