// dc_gemm_tc.cu -- tcgen05 tensor-core path of the verified W8A8 GEMM (sm_100a).
//
// out[bz, i, j] = epilogue( sum_p X[bz, i, p] * Wt[bz, j, p] )
//
// Swap-AB: the MMA's 128-row "M" side is 128 weight rows (= 128 output
// columns j), its "N" side is BN activation rows i (BN in {16..256}), so the
// small-M shapes of chunked prefill (M = 16) and lookahead waste no tensor
// work on padding rows of the weight.  Operands are K-major int8 tiles of
// 128 bytes of K, brought into shared memory by TMA with the 128-byte swizzle
// (no multicast), consumed by tcgen05.mma.cta_group::1.kind::i8 with int32
// accumulators in TMEM; the epilogue reads TMEM with tcgen05.ld and applies
// the verified epilogue f32(f32(f32(acc)*rs[i])*cs[j]) / ReLU / requant LUT
// (public/verified_core.js:227-228, 241-266).
//
// Roles: warp 0 lane 0 issues TMA, warp 1 lane 0 issues MMAs, warp 1 owns
// the TMEM allocation, and every warp runs the epilogue: warp w reads TMEM
// lanes 32(w%4)..32(w%4)+31 (its 32 output columns j) and, with more than four
// warps, one slice of the BN activation rows (128 threads for BN <= 16, 256 for
// BN = 32, 512 above: the epilogue of a 128 x 256 tile is 32K outputs, too much
// latency for four warps).  A STAGES-deep ring of full/empty mbarriers
// pipelines the loads against the MMAs.
//
// Split-K: when the output tiles do not fill the GPU, K is split across CTAs.
// Each split adds its int32 partial sums into a zeroed int32 scratch buffer
// with atomicAdd (integer addition is exact in any order); the last split to
// finish a tile (an atomic tile counter) applies the epilogue and resets the
// scratch and the counter to zero for the next call.
//
// Every wait on an mbarrier is bounded (%globaltimer, 2 s); a wait that gives
// up sets DC_ST_TIMEOUT in the context status word and the CTA winds down.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "dc_internal.cuh"

namespace {

constexpr int TILE_N = 128;   // weight rows (output columns) per CTA = MMA M
constexpr int TILE_K = 128;   // bytes of K per stage = one 128B swizzle row
constexpr int MMA_K = 32;     // K per tcgen05.mma of kind::i8
constexpr uint64_t WAIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try(bar, parity)) {
    if (gtimer() - t0 > WAIT_NS) {
      atomicOr(status, DC_ST_TIMEOUT);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// tma_load_2d with an L2 cache policy (evict-first for tiles no other CTA reads).
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_w(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                           bool once, uint64_t policy) {
  if (once)
    tma_load_2d_hint(dst, map, x, y, bar, policy);
  else
    tma_load_2d(dst, map, x, y, bar);
}
// UMMA shared-memory descriptor: K-major, 128B swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc(const void* p) {
  uint64_t d = (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;           // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32; // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;           // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;           // SWIZZLE_128B
  return d;
}
// Instruction descriptor of kind::i8: s8 x s8 -> s32, both K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t idesc_i8() {
  return (2u << 4)                       // D format: s32
         | (1u << 7) | (1u << 10)         // A, B: signed 8-bit
         | ((uint32_t)(BN >> 3) << 17)    // N >> 3
         | ((uint32_t)(TILE_N >> 4) << 24);  // M >> 4
}
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BN>
struct TcCfg {
  // BN <= 32 (chunked prefill): 5 stages (~92-102 KB), two CTAs per SM, so a
  // layer's tiles (up to ~296 CTAs) run in one wave
  static constexpr int STAGES = BN <= 32 ? 5 : (BN <= 64 ? 7 : (BN <= 128 ? 5 : 4));
  static constexpr int PER_SM = BN <= 32 ? 2 : 1;
  static constexpr int A_BYTES = TILE_N * TILE_K;
  static constexpr int B_BYTES = BN * TILE_K;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int THREADS = BN <= 16 ? 128 : (BN == 32 ? 256 : 512);
  static constexpr int COLS_PER_WARP = BN / (THREADS / 128);  // activation rows each epilogue warp covers
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

struct TcArgs {
  const float* rs;
  const float* cs;
  int m, k, n;
  int kb_total, kb_per_split, splits, m_tiles, n_tiles;
  unsigned flags;
  const int8_t* requant;
  const int8_t* relu;
  void* out;
  int32_t* partial;   // split-K int32 scratch (zero between calls), or null
  int* counters;      // split-K tile counters (zero between calls), or null
  int* status;
  int batch;          // k_gemm_tp2: batches its pairs loop over (its grid has one z slice)
};

// The epilogue of one CTA's 128 output columns j0.. x BN activation rows i0..:
// every warp reads TMEM lanes 32(w%4).. (its 32 columns) and COLS activation
// rows, applies the verified epilogue (or, split over K, adds its int32
// partial sums into the scratch and the last split to arrive finishes the
// tile, `tile` indexing its counter).  rs_s holds the BN row scales.
template <int BN, int COLS>
__device__ __forceinline__ void tc_epilogue(const TcArgs& a, uint32_t tmem, bool good, int bz, int j0, int i0,
                                            int tile, const float* rs_s) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3;                          // TMEM lanes 32*quarter .. +31
  const int cb0 = (warp >> 2) * COLS;        // this warp's activation rows
  const int cb1 = cb0 + COLS;
  const int j = j0 + quarter * 32 + lane;
  const bool jv = j < a.n;
  const float csv = jv ? __ldg(a.cs + bz * a.n + j) : 0.0f;
  // 16 accumulators of one column j (activation rows i0 + cbase ..): one
  // loop per output mode, walking the rows at a stride of n through a
  // pointer; residual values are all loaded before the first store
  const int64_t n64 = a.n;
  const bool relu = (a.flags & DC_RELU) != 0;
  auto store16 = [&](int cbase, const int32_t (&v)[16]) {
    const int cn = min(16, a.m - (i0 + cbase));
    if (!jv || cn <= 0) return;
    const int64_t base = ((int64_t)bz * a.m + i0 + cbase) * n64 + j;
    if (a.flags & DC_ACC) {  // (DC_ACC before DC_REQUANT, as dc_store_out)
      int32_t* o = (int32_t*)a.out + base;
#pragma unroll
      for (int c = 0; c < 16; c++)
        if (c < cn) o[(int64_t)c * n64] = v[c];
    } else if (a.flags & DC_REQUANT) {
      int8_t* o = (int8_t*)a.out + base;
#pragma unroll
      for (int c = 0; c < 16; c++)
        if (c < cn) o[(int64_t)c * n64] = dc_requant_unit(v[c], relu);
    } else {
      float* o = (float*)a.out + base;
      float old[16];
      if (a.flags & DC_F_ADDTO) {
#pragma unroll
        for (int c = 0; c < 16; c++) old[c] = c < cn ? o[(int64_t)c * n64] : 0.0f;
      }
#pragma unroll
      for (int c = 0; c < 16; c++) {
        if (c >= cn) continue;
        float x = dc_epi(v[c], rs_s[cbase + c], csv);
        if (relu && x < 0.0f) x = 0.0f;
        if (a.flags & DC_F_ADDTO) x = __fadd_rn(old[c], x);
        o[(int64_t)c * n64] = x;
      }
    }
  };
  if (a.splits == 1) {
    if (good) {
#pragma unroll 1
      for (int c0 = cb0; c0 < cb1; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, r);
        int32_t v[16];
#pragma unroll
        for (int c = 0; c < 16; c++) v[c] = (int32_t)r[c];
        store16(c0, v);
      }
    }
  } else {
    if (good) {
#pragma unroll 1
      for (int c0 = cb0; c0 < cb1; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, r);
#pragma unroll
        for (int c = 0; c < 16; c++) {
          const int i = i0 + c0 + c;
          if (jv && i < a.m) atomicAdd(a.partial + ((int64_t)bz * a.m + i) * a.n + j, (int32_t)r[c]);
        }
      }
    }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) last = (atomicAdd(a.counters + tile, 1) == a.splits - 1);
    __syncthreads();
    if (last) {
      __threadfence();
#pragma unroll 1
      for (int c0 = cb0; c0 < cb1; c0 += 16) {
        int32_t v[16];
#pragma unroll
        for (int c = 0; c < 16; c++) {  // all 16 partial sums in flight together
          const int i = i0 + c0 + c;
          v[c] = (jv && i < a.m) ? __ldcg(a.partial + ((int64_t)bz * a.m + i) * a.n + j) : 0;
        }
        store16(c0, v);
#pragma unroll
        for (int c = 0; c < 16; c++) {
          const int i = i0 + c0 + c;
          if (jv && i < a.m) a.partial[((int64_t)bz * a.m + i) * a.n + j] = 0;
        }
      }
      if (threadIdx.x == 0) a.counters[tile] = 0;
    }
  }

}

template <int BN>
__global__ void __launch_bounds__(TcCfg<BN>::THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const TcArgs a) {
  using C = TcCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = (uint64_t*)(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = (uint32_t*)(accum + 1);
  int* flag = (int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile_n = blockIdx.x, tile_m = blockIdx.y;
  const int bz = blockIdx.z / a.splits, split = blockIdx.z - bz * a.splits;
  const int j0 = tile_n * TILE_N, i0 = tile_m * BN;
  const int kb0 = split * a.kb_per_split;
  const int kb1 = min(a.kb_total, kb0 + a.kb_per_split);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    *flag = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer.  Launched as a programmatic dependent: the weight
    // tiles of the first stages (constant data) are requested before the
    // grid-dependency wait, the activation tiles (written by the previous
    // kernel) after it.
    int issued = 0;
    bool ok = true;
    // with a single row tile every weight tile is read by exactly one CTA
    const bool once = gridDim.y == 1;
    uint64_t pol = 0;
    if (once) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    const int pre = min(nkb, C::STAGES);
    for (int it = 0; it < pre; it++) {
      mbar_expect_tx(&full[it], C::STAGE_BYTES);
      tma_load_w(sA + it * C::A_BYTES, &tmW, (kb0 + it) * TILE_K, bz * a.n + j0, &full[it], once, pol);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int it = 0; it < pre; it++)
      tma_load_2d(sB + it * C::B_BYTES, &tmX, (kb0 + it) * TILE_K, bz * a.m + i0, &full[it]);
    issued = pre;
    for (int it = pre; it < nkb && ok; it++) {
      const int s = it % C::STAGES;
      const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
      ok = mbar_wait(&empty[s], ph ^ 1u, a.status);
      if (!ok) break;
      mbar_expect_tx(&full[s], C::STAGE_BYTES);
      const int kx = (kb0 + it) * TILE_K;
      tma_load_w(sA + s * C::A_BYTES, &tmW, kx, bz * a.n + j0, &full[s], once, pol);
      tma_load_2d(sB + s * C::B_BYTES, &tmX, kx, bz * a.m + i0, &full[s]);
      issued++;
    }
    if (!ok) {
      // wind down: let every issued load land before the CTA's memory goes away
      atomicExch(flag, 1);
      for (int it = max(0, issued - C::STAGES); it < issued; it++)
        mbar_wait(&full[it % C::STAGES], (uint32_t)(it / C::STAGES) & 1u, a.status);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    const uint32_t idesc = idesc_i8<BN>();
    for (int it = 0; it < nkb; it++) {
      const int s = it % C::STAGES;
      const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
      if (!mbar_wait(&full[s], ph, a.status)) { atomicExch(flag, 1); break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint8_t* ta = sA + s * C::A_BYTES;
      const uint8_t* tb = sB + s * C::B_BYTES;
#pragma unroll
      for (int kk = 0; kk < TILE_K / MMA_K; kk++)
        mma_i8(tmem, umma_desc(ta + kk * MMA_K), umma_desc(tb + kk * MMA_K), idesc, (it > 0 || kk > 0) ? 1u : 0u);
      mma_commit(&empty[s]);  // the slot is free once these MMAs have read it
    }
    mma_commit(accum);  // all MMAs issued by this thread are complete
  }
  __syncwarp();

  // ---- epilogue (all four warps); rs and a residual `out` come from earlier kernels
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the tile's row scales, once, into shared memory (the stores below may
  // alias them as far as the compiler knows, which would serialise every load)
  __shared__ float rs_s[BN];
  for (int c = threadIdx.x; c < BN; c += blockDim.x) rs_s[c] = (i0 + c < a.m) ? __ldg(a.rs + bz * a.m + i0 + c) : 0.0f;
  const bool have = mbar_wait(accum, 0, a.status);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();
  const bool good = have && (*(volatile int*)flag == 0) && nkb > 0;
  tc_epilogue<BN, C::COLS_PER_WARP>(a, tmem, good, bz, j0, i0, (bz * a.m_tiles + tile_m) * a.n_tiles + tile_n, rs_s);

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
  }
}

// ---- the 2-SM variant for M > 128 -------------------------------------------
// A CTA pair (a cluster of two along x) computes one 256 x 256 tile: 256
// weight rows (this CTA's 128 at j0) against 256 activation rows (i0..), with
// tcgen05.mma.cta_group::2 (M = 256, N = 256) issued by the pair's even CTA.
// Each CTA brings its own 128 weight rows and 128 of the 256 activation rows
// of every K block into its shared memory (TMA with .cta_group::2, no
// multicast; the copies of both CTAs complete on the even CTA's `full`
// barrier); the MMA reads the two halves from the two CTAs, and its commits
// are multicast to both CTAs' `empty` and `accum` barriers.  A stage is then
// 32 KB per CTA instead of 48, so six stages fit where one CTA held four:
// about 2.5 us of MMA work in flight against the TMA round trip.  Each CTA's
// TMEM holds its 128 weight rows x 256 activation rows; the epilogue is
// tc_epilogue's.  Every wait is bounded; every path of both CTAs reaches the
// closing cluster barrier before the pair frees its TMEM.
constexpr int TC2_STAGES = 6;
constexpr int TC2_HALF = 128 * TILE_K;  // 16 KB: 128 rows of one operand
constexpr int TC2_STAGE = 2 * TC2_HALF;
constexpr int TC2_SMEM = TC2_STAGES * TC2_STAGE + 1024 + 256;
constexpr int TC2_THREADS = 512;
constexpr int TC2_COLS = 256 / (TC2_THREADS / 128);

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 2-D tile load into this CTA's shared memory, completing on the barrier at
// cluster address `bar` (the even CTA's), as one half of a pair's operand.
__device__ __forceinline__ void tma_load_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_i8_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` in both CTAs of the pair once the MMAs issued so far are done.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

__global__ void __launch_bounds__(TC2_THREADS, 1)
    k_gemm_tc2(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;                            // STAGES x 16 KB: this CTA's 128 weight rows
  uint8_t* sB = smem + TC2_STAGES * TC2_HALF;    // STAGES x 16 KB: this CTA's 128 activation rows
  uint64_t* full = (uint64_t*)(smem + TC2_STAGES * TC2_STAGE);
  uint64_t* empty = full + TC2_STAGES;
  uint64_t* accum = empty + TC2_STAGES;
  uint32_t* tmem_slot = (uint32_t*)(accum + 1);
  int* flag = (int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int tile_n = blockIdx.x >> 1, tile_m = blockIdx.y;
  const int bz = blockIdx.z / a.splits, split = blockIdx.z - bz * a.splits;
  const int j0 = tile_n * 256 + 128 * (int)rank;  // this CTA's weight rows = output columns
  const int i0 = tile_m * 256;                    // the pair's activation rows
  const int kb0 = split * a.kb_per_split;
  const int kb1 = min(a.kb_total, kb0 + a.kb_per_split);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC2_STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    *flag = 0;
  }
  if (warp == 1) {  // the same warp in both CTAs allocates the pair's TMEM
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(256u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync_all();  // both CTAs' barriers exist before any copy or commit reaches them
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer, both CTAs.  Weights (constant) first, before the
    // grid-dependency wait; activations after it.
    const uint32_t full_l = map_rank(&full[0], 0);  // the even CTA's barriers
    bool ok = true;
    const int pre = min(nkb, TC2_STAGES);
    for (int it = 0; it < pre; it++) {
      if (leader) mbar_expect_tx(&full[it], 2 * TC2_STAGE);  // both CTAs' halves of both operands
      tma_load_pair(sA + it * TC2_HALF, &tmW, (kb0 + it) * TILE_K, bz * a.n + j0, full_l + 8 * it);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int it = 0; it < pre; it++)
      tma_load_pair(sB + it * TC2_HALF, &tmX, (kb0 + it) * TILE_K, bz * a.m + i0 + 128 * (int)rank, full_l + 8 * it);
    for (int it = pre; it < nkb && ok; it++) {
      const int s = it % TC2_STAGES;
      const uint32_t ph = (uint32_t)(it / TC2_STAGES) & 1u;
      ok = mbar_wait(&empty[s], ph ^ 1u, a.status);
      if (!ok) break;
      if (leader) mbar_expect_tx(&full[s], 2 * TC2_STAGE);
      const int kx = (kb0 + it) * TILE_K;
      tma_load_pair(sA + s * TC2_HALF, &tmW, kx, bz * a.n + j0, full_l + 8 * s);
      tma_load_pair(sB + s * TC2_HALF, &tmX, kx, bz * a.m + i0 + 128 * (int)rank, full_l + 8 * s);
    }
    if (!ok) atomicExch(flag, 1);
  } else if (warp == 1 && lane == 0 && leader) {
    // ---- MMA issuer (the even CTA only)
    const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
                           ((uint32_t)(256 >> 4) << 24);  // s8 x s8 -> s32, K-major, M = 256, N = 256
    int done = 0;
    for (int it = 0; it < nkb; it++) {
      const int s = it % TC2_STAGES;
      const uint32_t ph = (uint32_t)(it / TC2_STAGES) & 1u;
      if (!mbar_wait(&full[s], ph, a.status)) {
        atomicExch(flag, 1);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint8_t* ta = sA + s * TC2_HALF;
      const uint8_t* tb = sB + s * TC2_HALF;
#pragma unroll
      for (int kk = 0; kk < TILE_K / MMA_K; kk++)
        mma_i8_pair(tmem, umma_desc(ta + kk * MMA_K), umma_desc(tb + kk * MMA_K), idesc,
                    (it > 0 || kk > 0) ? 1u : 0u);
      mma_commit_pair(&empty[s]);
      done = it + 1;
    }
    mma_commit_pair(accum);
    // after an abort: every stage issued but not consumed lands before the pair goes away
    for (int it = done; it < min(nkb, done + TC2_STAGES); it++)
      mbar_wait(&full[it % TC2_STAGES], (uint32_t)(it / TC2_STAGES) & 1u, a.status);
  }
  __syncwarp();

  // ---- epilogue (both CTAs, all warps)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float rs_s[256];
  for (int c = threadIdx.x; c < 256; c += blockDim.x) rs_s[c] = (i0 + c < a.m) ? __ldg(a.rs + bz * a.m + i0 + c) : 0.0f;
  const bool have = mbar_wait(accum, 0, a.status);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();
  // either CTA's failure spoils the pair's tile: read the other CTA's flag too
  cluster_sync_all();
  int bad = *(volatile int*)flag;
  {
    uint32_t other;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(other) : "r"(map_rank(flag, rank ^ 1u)));
    bad |= (int)other;
  }
  const bool good = have && bad == 0 && nkb > 0;
  tc_epilogue<256, TC2_COLS>(a, tmem, good, bz, j0, i0, (bz * a.m_tiles + tile_m) * a.n_tiles + 2 * tile_n + rank,
                             rs_s);

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();  // neither CTA frees the pair's TMEM or leaves while the other still uses it
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256u) : "memory");
  }
}

// ---- the persistent 2-SM variant ---------------------------------------------
// k_gemm_tc2's tiles and operand split, with each CTA pair looping over pair
// tiles t = pair, pair + pairs, ... (the activation-tile index fastest, so the
// pairs running together share weight tiles through L2) and a double-buffered
// accumulator: the pair's TMEM holds two 256-column accumulators, the even
// CTA's MMA thread fills one while the epilogue warps of both CTAs drain the
// other.  The epilogue warps hand a buffer back with a remote arrive on the
// even CTA's `tempty` barrier.  Warps: 0 TMA producer, 1 MMA issuer (even CTA)
// and TMEM owner, 2-3 idle, 4-11 epilogue (two per TMEM lane quarter, 128
// activation rows each).  No split-K: used when the pair tiles fill the SMs.
constexpr int TP2_THREADS = 384;
constexpr int TP2_EPI_WARPS = 8;
constexpr int TP2_SMEM = TC2_STAGES * TC2_STAGE + 1024 + 512 + 2 * 256 * 4;

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__global__ void __launch_bounds__(TP2_THREADS, 1)
    k_gemm_tp2(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + TC2_STAGES * TC2_HALF;
  uint64_t* full = (uint64_t*)(smem + TC2_STAGES * TC2_STAGE);
  uint64_t* empty = full + TC2_STAGES;
  uint64_t* tfull = empty + TC2_STAGES;  // [2]: an accumulator is complete
  uint64_t* tempty = tfull + 2;          // [2]: an accumulator is drained (the even CTA's count both CTAs)
  uint32_t* tmem_slot = (uint32_t*)(tempty + 2);
  int* flag = (int*)(tmem_slot + 1);
  float* rs_s = (float*)(smem + TC2_STAGES * TC2_STAGE + 512);  // [2][256]: a tile's row scales (f32 output)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  if (warp == 0 && lane == 0) {  // the descriptors' first fetch overlaps the set-up
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmW) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmX) : "memory");
  }
  const int pairs_n = a.n_tiles >> 1;
  const int tiles = pairs_n * a.m_tiles * a.batch;
  const int nkb = a.kb_total;
  // pair tile t -> (bz, tile_m, tile_n), tile_m fastest
  auto decode = [&](int t, int& bz, int& tm, int& tn) {
    tm = t % a.m_tiles;
    tn = (t / a.m_tiles) % pairs_n;
    bz = t / (a.m_tiles * pairs_n);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC2_STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * TP2_EPI_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    *flag = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer, both CTAs, one K-block stream across all its tiles
    const uint32_t full_l = map_rank(&full[0], 0);
    int it = 0;
    bool waited = false;
    for (int t = pair; t < tiles && !*(volatile int*)flag; t += pairs) {
      int bz, tm, tn;
      decode(t, bz, tm, tn);
      const int j0 = tn * 256 + 128 * (int)rank, i0 = tm * 256 + 128 * (int)rank;
      for (int kb = 0; kb < nkb; kb++, it++) {
        const int s = it % TC2_STAGES;
        if (it >= TC2_STAGES && !mbar_wait(&empty[s], ((uint32_t)(it / TC2_STAGES) & 1u) ^ 1u, a.status)) {
          atomicExch(flag, 1);
          break;
        }
        if (leader) mbar_expect_tx(&full[s], 2 * TC2_STAGE);
        tma_load_pair(sA + s * TC2_HALF, &tmW, kb * TILE_K, bz * a.n + j0, full_l + 8 * s);
        if (!waited) {  // activations come from the kernel before this one
          asm volatile("griddepcontrol.wait;" ::: "memory");
          waited = true;
        }
        tma_load_pair(sB + s * TC2_HALF, &tmX, kb * TILE_K, bz * a.m + i0, full_l + 8 * s);
      }
    }
    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
  } else if (warp == 1 && lane == 0 && leader) {
    // ---- MMA issuer (the even CTA)
    const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
                           ((uint32_t)(256 >> 4) << 24);
    int it = 0, lt = 0;
    bool ok = true;
    for (int t = pair; t < tiles && ok; t += pairs, lt++) {
      const int b = lt & 1, use = lt >> 1;
      if (use > 0 && !mbar_wait(&tempty[b], (uint32_t)(use - 1) & 1u, a.status)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t acc = tmem + (uint32_t)(b * 256);
      for (int kb = 0; kb < nkb; kb++, it++) {
        const int s = it % TC2_STAGES;
        if (!mbar_wait(&full[s], (uint32_t)(it / TC2_STAGES) & 1u, a.status)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint8_t* ta = sA + s * TC2_HALF;
        const uint8_t* tb = sB + s * TC2_HALF;
#pragma unroll
        for (int kk = 0; kk < TILE_K / MMA_K; kk++)
          mma_i8_pair(acc, umma_desc(ta + kk * MMA_K), umma_desc(tb + kk * MMA_K), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit_pair(&empty[s]);
      }
      mma_commit_pair(&tfull[b]);  // (after an abort too: the epilogues wake and see the flag)
    }
    if (!ok) {
      atomicExch(flag, 1);
      // every stage issued but not consumed lands before the pair goes away
      for (int k = it; k < it + TC2_STAGES; k++) mbar_wait(&full[k % TC2_STAGES], (uint32_t)(k / TC2_STAGES) & 1u, a.status);
    }
  } else if (warp >= 4) {
    // ---- epilogue warps, both CTAs.  Each thread owns one output column j and
    // walks 128 activation rows at a stride of n through a pointer; the modes
    // are separate loops, so the int8 / int32 outputs read nothing but TMEM and
    // the f32 output reads its row scales from shared memory (staged once per
    // tile), never a global load between two stores.
    asm volatile("griddepcontrol.wait;" ::: "memory");  // rs and a residual `out` come from earlier kernels
    const int quarter = warp & 3, part = (warp - 4) >> 2;  // TMEM lanes 32*quarter.., activation rows part*128..
    const int et = threadIdx.x - 128;                      // 0..255 over the epilogue warps
    const uint32_t tempty_l = map_rank(&tempty[0], 0);
    const bool f32_out = !(a.flags & (DC_ACC | DC_REQUANT));
    const bool relu = (a.flags & DC_RELU) != 0, addto = (a.flags & DC_F_ADDTO) != 0;
    const int64_t n64 = a.n;
    int lt = 0;
    for (int t = pair; t < tiles; t += pairs, lt++) {
      const int b = lt & 1, use = lt >> 1;
      int bz, tm, tn;
      decode(t, bz, tm, tn);
      float* rsb = rs_s + b * 256;
      if (f32_out) {  // (double-buffered: a warp cannot pass the next tile's barrier before all leave this one)
        const int i = tm * 256 + et;
        rsb[et] = i < a.m ? __ldg(a.rs + (int64_t)bz * a.m + i) : 0.0f;
        asm volatile("bar.sync 1, 256;" ::: "memory");
      }
      // every epilogue warp takes every tile of the loop (so all meet at each
      // barrier above); after a failure they only hand the buffers back
      const bool have = !*(volatile int*)flag && mbar_wait(&tfull[b], (uint32_t)use & 1u, a.status);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (!have) atomicExch(flag, 1);
      if (have && !*(volatile int*)flag) {
        const int j = tn * 256 + 128 * (int)rank + quarter * 32 + lane;
        const int i0 = tm * 256 + part * 128;
        const int rows = min(128, a.m - i0);  // activation rows of this warp in range (<= 0: none)
        const bool jv = j < a.n;
        const float csv = (f32_out && jv) ? __ldg(a.cs + (int64_t)bz * a.n + j) : 0.0f;
        const int64_t base = ((int64_t)bz * a.m + i0) * n64 + j;
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 256 + part * 128);
#pragma unroll 1
        for (int c0 = 0; c0 < 128 && c0 < rows; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + (uint32_t)c0, r);
          if (!jv) continue;
          const int cn = min(16, rows - c0);
          if (a.flags & DC_ACC) {  // (DC_ACC before DC_REQUANT, as dc_store_out)
            int32_t* o = (int32_t*)a.out + base + (int64_t)c0 * n64;
#pragma unroll
            for (int c = 0; c < 16; c++)
              if (c < cn) o[(int64_t)c * n64] = (int32_t)r[c];
          } else if (a.flags & DC_REQUANT) {
            int8_t* o = (int8_t*)a.out + base + (int64_t)c0 * n64;
#pragma unroll
            for (int c = 0; c < 16; c++)
              if (c < cn) o[(int64_t)c * n64] = dc_requant_unit((int32_t)r[c], relu);
          } else {
            float* o = (float*)a.out + base + (int64_t)c0 * n64;
            const float* rsv = rsb + part * 128 + c0;
            float old[16];
            if (addto) {  // all 16 residual loads in flight before the first store
#pragma unroll
              for (int c = 0; c < 16; c++) old[c] = c < cn ? o[(int64_t)c * n64] : 0.0f;
            }
#pragma unroll
            for (int c = 0; c < 16; c++) {
              if (c >= cn) continue;
              float v = dc_epi((int32_t)r[c], rsv[c], csv);
              if (relu && v < 0.0f) v = 0.0f;
              if (addto) v = __fadd_rn(old[c], v);
              o[(int64_t)c * n64] = v;
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty_l + 8 * b);  // this warp is done with buffer b
    }
  }
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();  // neither CTA frees the pair's TMEM or leaves while the other still uses it
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    else
      cudaGetLastError();
  }
  return fn;
}

// 2-D int8 map over `rows` rows of `ld` bytes, box = 128 bytes x box_rows, 128B swizzle.
// A map is a pure function of (address, ld, rows, box rows), so encoded maps are
// cached under that key: the resident weights and the stage's activation
// buffers are encoded once instead of on every GEMM call.
struct MapKey {
  uintptr_t base;
  long rows;
  int ld, box;
  bool operator==(const MapKey& o) const { return base == o.base && rows == o.rows && ld == o.ld && box == o.box; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.base) ^ (std::hash<long>()(k.rows) * 31u) ^ ((size_t)k.ld << 20) ^ (size_t)k.box;
  }
};
std::mutex g_map_lock;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

bool encode_map(CUtensorMap* map, const void* base, int ld, long rows, int box_rows);

bool make_map(CUtensorMap* map, const void* base, int ld, long rows, int box_rows) {
  const MapKey key{(uintptr_t)base, rows, ld, box_rows};
  std::lock_guard<std::mutex> guard(g_map_lock);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *map = it->second;
    return true;
  }
  if (!encode_map(map, base, ld, rows, box_rows)) return false;
  if (g_maps.size() > 65536) g_maps.clear();
  g_maps.emplace(key, *map);
  return true;
}

bool encode_map(CUtensorMap* map, const void* base, int ld, long rows, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)TILE_K, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN>
int launch_tc(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs, const float* cs,
              int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st, int32_t* partial,
              int* counters, size_t partial_cap, size_t counter_cap, int clear) {
  using C = TcCfg<BN>;
  CUtensorMap mW, mX;
  if (!make_map(&mW, Wt, ldw, (long)batch * n, TILE_N) || !make_map(&mX, Xq, ldx, (long)batch * m, BN))
    return dc_fail(ctx, DC_E_INVAL, "tcgen05: tensor map encode failed");
  TcArgs a;
  a.rs = rs;
  a.cs = cs;
  a.m = m;
  a.k = k;
  a.n = n;
  a.kb_total = (k + TILE_K - 1) / TILE_K;
  a.n_tiles = (n + TILE_N - 1) / TILE_N;
  a.m_tiles = (m + BN - 1) / BN;
  const int tiles = a.n_tiles * a.m_tiles * batch;
  int splits = 1;
  const int slots = ctx->sm_count * C::PER_SM;  // CTAs resident at once
  if (tiles < slots && a.kb_total > 1) {
    splits = slots / tiles;  // the whole grid in one wave
    // at least 4 K blocks (512 bytes of K) per split: a CTA's fixed costs
    // (TMEM allocation, pipeline fill, the split-K fixup) need work to hide behind
    splits = std::min(splits, std::max(1, a.kb_total / 4));
    if (splits > a.kb_total) splits = a.kb_total;
  }
  a.kb_per_split = (a.kb_total + splits - 1) / splits;
  splits = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  if (splits > 1 && (!partial || (size_t)batch * m * n > partial_cap || (size_t)tiles > counter_cap)) {
    splits = 1;
    a.kb_per_split = a.kb_total;
  }
  a.splits = splits;
  if (splits > 1 && clear) {  // caller-owned scratch of unknown contents: zero what the split-K fixup reads
    DC_CUDA(ctx, cudaMemsetAsync(partial, 0, 4 * (size_t)batch * m * n, st));
    DC_CUDA(ctx, cudaMemsetAsync(counters, 0, 4 * (size_t)tiles, st));
  }
  a.flags = flags;
  a.requant = ctx->d_requant;
  a.relu = ctx->d_relu;
  a.out = out;
  a.partial = partial;
  a.counters = counters;
  a.status = ctx->d_status;
  if (int rc = dc_set_smem(ctx, (const void*)k_gemm_tc<BN>, C::SMEM)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_tiles, a.m_tiles, batch * splits);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DC_CUDA(ctx, cudaLaunchKernelEx(&cfg, k_gemm_tc<BN>, mW, mX, a));
  dc_count_launch();
  return DC_OK;
}

// k_gemm_tc2 over pairs of SMs: grid (2 * ceil(n/256), ceil(m/256), batch * splits), clusters of two.
int launch_tc2(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs, const float* cs,
               int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st, int32_t* partial,
               int* counters, size_t partial_cap, size_t counter_cap, int clear) {
  CUtensorMap mW, mX;
  if (!make_map(&mW, Wt, ldw, (long)batch * n, TILE_N) || !make_map(&mX, Xq, ldx, (long)batch * m, 128))
    return dc_fail(ctx, DC_E_INVAL, "tcgen05: tensor map encode failed");
  TcArgs a;
  a.rs = rs;
  a.cs = cs;
  a.m = m;
  a.k = k;
  a.n = n;
  a.kb_total = (k + TILE_K - 1) / TILE_K;
  const int pairs_n = (n + 255) / 256;
  a.n_tiles = 2 * pairs_n;  // 128-column slots (the split-K counters' index)
  a.m_tiles = (m + 255) / 256;
  const int ctas = 2 * pairs_n * a.m_tiles * batch;
  int splits = 1;
  if (ctas < ctx->sm_count && a.kb_total > 1) {
    splits = std::max(1, ctx->sm_count / ctas);
    splits = std::min(splits, std::max(1, a.kb_total / 4));
  }
  a.kb_per_split = (a.kb_total + splits - 1) / splits;
  splits = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  const size_t tiles = (size_t)a.n_tiles * a.m_tiles * batch;
  if (splits > 1 && (!partial || (size_t)batch * m * n > partial_cap || tiles > counter_cap)) {
    splits = 1;
    a.kb_per_split = a.kb_total;
  }
  a.splits = splits;
  if (splits > 1 && clear) {
    DC_CUDA(ctx, cudaMemsetAsync(partial, 0, 4 * (size_t)batch * m * n, st));
    DC_CUDA(ctx, cudaMemsetAsync(counters, 0, 4 * tiles, st));
  }
  a.flags = flags;
  a.requant = ctx->d_requant;
  a.relu = ctx->d_relu;
  a.out = out;
  a.partial = partial;
  a.counters = counters;
  a.status = ctx->d_status;
  if (int rc = dc_set_smem(ctx, (const void*)k_gemm_tc2, TC2_SMEM)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs_n, a.m_tiles, batch * splits);
  cfg.blockDim = dim3(TC2_THREADS);
  cfg.dynamicSmemBytes = TC2_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  DC_CUDA(ctx, cudaLaunchKernelEx(&cfg, k_gemm_tc2, mW, mX, a));
  dc_count_launch();
  return DC_OK;
}

// k_gemm_tp2: as many CTA pairs as fit beside each other (at most one per two
// SMs), each looping over its share of the pair tiles.
int launch_tp2(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs, const float* cs,
               int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st) {
  CUtensorMap mW, mX;
  if (!make_map(&mW, Wt, ldw, (long)batch * n, TILE_N) || !make_map(&mX, Xq, ldx, (long)batch * m, 128))
    return dc_fail(ctx, DC_E_INVAL, "tcgen05: tensor map encode failed");
  TcArgs a = {};
  a.rs = rs;
  a.cs = cs;
  a.m = m;
  a.k = k;
  a.n = n;
  a.kb_total = (k + TILE_K - 1) / TILE_K;
  a.kb_per_split = a.kb_total;
  a.splits = 1;
  a.n_tiles = 2 * ((n + 255) / 256);
  a.m_tiles = (m + 255) / 256;
  a.batch = batch;
  a.flags = flags;
  a.requant = ctx->d_requant;
  a.relu = ctx->d_relu;
  a.out = out;
  a.status = ctx->d_status;
  const int tiles = (a.n_tiles / 2) * a.m_tiles * batch;
  const int pairs = std::max(1, std::min(ctx->sm_count / 2, tiles));
  if (int rc = dc_set_smem(ctx, (const void*)k_gemm_tp2, TP2_SMEM)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(TP2_THREADS);
  cfg.dynamicSmemBytes = TP2_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  DC_CUDA(ctx, cudaLaunchKernelEx(&cfg, k_gemm_tp2, mW, mX, a));
  dc_count_launch();
  return DC_OK;
}

}  // namespace

// Split-K scratch of a context: int32 partial sums and tile counters, both kept
// at zero between calls by the kernel itself.
static int tc_scratch(dc_ctx* ctx, size_t partial_elems, size_t counters, int32_t** p, int** c) {
  if (partial_elems > ctx->tc_partial_cap || counters > ctx->tc_counter_cap) {
    DC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(ctx->tc_partial);
    cudaFree(ctx->tc_counters);
    ctx->tc_partial = nullptr;
    ctx->tc_counters = nullptr;
    ctx->tc_partial_cap = ctx->tc_counter_cap = 0;
    size_t pe = partial_elems > (1u << 20) ? partial_elems : (1u << 20);
    size_t ce = counters > 4096 ? counters : 4096;
    if (cudaMalloc(&ctx->tc_partial, pe * 4) != cudaSuccess || cudaMalloc(&ctx->tc_counters, ce * 4) != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(ctx, DC_E_NOMEM, "split-K scratch allocation failed");
    }
    DC_CUDA(ctx, cudaMemset(ctx->tc_partial, 0, pe * 4));
    DC_CUDA(ctx, cudaMemset(ctx->tc_counters, 0, ce * 4));
    ctx->tc_partial_cap = pe;
    ctx->tc_counter_cap = ce;
  }
  *p = ctx->tc_partial;
  *c = ctx->tc_counters;
  return DC_OK;
}

int dc_gemm_tc_with(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                    const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st,
                    int32_t* partial, int* counters, size_t partial_cap, size_t counter_cap, int clear) {
  if (((uintptr_t)Xq & 15) || ((uintptr_t)Wt & 15) || (ldx & 15) || (ldw & 15) || k <= 0 || m <= 0 || n <= 0)
    return dc_fail(ctx, DC_E_INVAL, "tcgen05: operands must be 16-byte aligned with ld a multiple of 16");
  if (m <= 16)
    return launch_tc<16>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, partial, counters,
                         partial_cap, counter_cap, clear);
  if (m <= 32)
    return launch_tc<32>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, partial, counters,
                         partial_cap, counter_cap, clear);
  if (m <= 64)
    return launch_tc<64>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, partial, counters,
                         partial_cap, counter_cap, clear);
  if (m <= 128)
    return launch_tc<128>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, partial, counters,
                          partial_cap, counter_cap, clear);
  // enough pair tiles to give every SM pair one: the persistent kernel
  // up to 512 rows with too few 256 x 256 tile pairs to fill half the SMs: 1-SM
  // tiles of 128 rows (four times the CTAs, split-K over the rest)
  if (m <= 512 && (size_t)((n + 255) / 256) * ((m + 255) / 256) * batch < (size_t)ctx->sm_count / 2)
    return launch_tc<128>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, partial, counters,
                          partial_cap, counter_cap, clear);
  if (ctx->tc2_enabled && ctx->tp2_enabled &&
      (size_t)((n + 255) / 256) * ((m + 255) / 256) * batch >= (size_t)ctx->sm_count / 2)
    return launch_tp2(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st);
  if (ctx->tc2_enabled)
    return launch_tc2(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, partial, counters, partial_cap,
                      counter_cap, clear);
  return launch_tc<256>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, partial, counters,
                        partial_cap, counter_cap, clear);
}

int dc_gemm_tc(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs, const float* cs,
               int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st) {
  int32_t* partial = nullptr;
  int* counters = nullptr;
  // worst case over the BN choices: tiles = ceil(n/128) * ceil(m/16) * batch
  size_t tiles = (size_t)((n + 127) / 128) * ((m + 15) / 16) * batch;
  int rc = tc_scratch(ctx, (size_t)batch * m * n, tiles, &partial, &counters);
  if (rc) return rc;
  return dc_gemm_tc_with(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, partial, counters,
                         ctx->tc_partial_cap, ctx->tc_counter_cap, 0);
}
