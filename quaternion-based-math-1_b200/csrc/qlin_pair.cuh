// Prefill-sized quaternion linear forward on a pair of SMs (sm_100a):
// persistent, 2-SM tcgen05 UMMA (cta_group::2) with the weight operand
// expanded into tensor memory.
//
// The layer is y = x Wd^T with the real block matrix
//
//     Wd[4o + a, 4i + q] = s(a, a^q) * W_{a^q}[o, i]
//
// (reference quaternion/packing.py:18-21 and quaternion/linear.py:66-69: row
// block a of the 4x4 block matrix holds W_{a^q} in column block q, negated
// where the table has a minus).  Wd is four times the weight bytes, so it is
// never stored anywhere: TMA brings W_p tiles (a quarter of a dense layer's
// weight traffic) into shared memory, the builder warps apply the component
// swap and the sign in registers and write the Wd rows of the current K
// stage into tensor memory with tcgen05.st, where the UMMA reads them as its
// A operand.  x is the B operand exactly as the caller stores it ([M, K]
// rows, K-major, loaded by TMA with 128-byte swizzling): no component planes,
// no prologue kernel.
//
// Tile of one CTA pair (a 2-CTA cluster): 256 real outputs (64 output
// quaternions; 128 rows of Wd in each CTA's tensor memory) x NTOK tokens
// (NTOK / 2 tokens of x in each CTA's shared memory).  One UMMA of M = 256,
// N = NTOK, K = 16 per step, issued by the pair's even CTA, reads A from both
// CTAs' tensor memory and B from both CTAs' shared memory and accumulates
// into both CTAs' tensor memory (each CTA's 128 rows).  Per SM and UMMA step
// the shared-memory traffic is the x half-tile written by TMA and read by the
// UMMA plus a small W tile (at most 80 B/clk at full tensor rate, of 128);
// the expanded weight operand costs tensor-memory stores, not shared memory.
//
// The issuing thread spends about 60-130 cycles on every tcgen05
// instruction, barrier wait and fence (measured), so the bookkeeping per
// stage is kept to one barrier wait and two commits around eight UMMAs, and
// the large tile (NTOK = 256, 128 cycles per UMMA) is the prefill shape:
// its single accumulator (256 columns) is drained into registers by the
// epilogue first and released before the stores, so the next tile's UMMAs
// wait only for that drain.  NTOK = 128 keeps two accumulators for smaller
// token counts.  Tensor memory (512 columns per CTA): the accumulator(s),
// then a 4-stage ring of expanded weight rows (64 columns = 32 input
// quaternions per stage).  Shared memory: a ring of x half-tiles and W tiles
// (4 stages at NTOK = 256, 8 at 128).  The pair walks the tiles
// tile = pair, pair + pairs, ... (persistent grid of one pair per two SMs).
//
// Roles (320 threads per CTA):
//   warp 0, lane 0   TMA producer of this CTA's x half-tiles and W tiles
//   warp 1           tensor-memory allocation (both CTAs); lane 0 of the even
//                    CTA issues the UMMAs
//   warps 2-5        builders: wait for their own CTA's stage (x and W), write
//                    expanded weight rows into tensor memory (warp w writes
//                    lanes 32 (w % 4) .. +31) and arrive on the even CTA's
//                    barrier -- so its one wait covers both CTAs' x and A
//   warps 6-9        epilogue: accumulator -> bias -> one rounding -> y
//                    (warp w reads lanes 32 (w % 4) .. +31)
// Tensor-memory lane 32 q + l of a CTA holds real output
// n0 + 32 q + 4 (l % 8) + l / 8 (output quaternion 8 q + l % 8, component
// l / 8), so that a builder warp's shared-memory reads of the swizzled W
// tiles are free of bank conflicts.
// Every mbarrier wait is bounded; a wait that runs out records
// QLIN_ERR_TIMEOUT, the CTA stops issuing work, and both CTAs still meet at
// the final cluster barrier and release their tensor memory.
#pragma once

#include <type_traits>

#include "qlin_common.cuh"

namespace qlin {

constexpr int kPairThreads = 320;
constexpr int kPairRows = 128;          // real outputs per CTA (UMMA M = 256 per pair)
constexpr int kPairStageK = 128;        // real inputs per stage (32 input quaternions)
constexpr int kPairAStages = 4;         // tensor-memory ring of expanded weight rows
constexpr int kPairWTileBytes = 32 * 64;                      // one component: 32 rows x 32 inputs
constexpr int kPairACols = kPairStageK / 2;                   // 64 tensor-memory columns per A stage
constexpr int kPairEpiTokens = 16;                            // tokens per epilogue store group
constexpr int kPairEpiBufBytes = kPairEpiTokens * kPairRows * 2;  // 4 KB staging (bf16/f16)
constexpr int kPairEpiBar = 2;                                // named barrier of the epilogue warps
constexpr int kPairSmemBytes = 204 * 1024;

template <int NTOK>
struct PairCfg {
  static_assert(NTOK == 128 || NTOK == 256, "pair tile tokens");
  static constexpr int kHalf = NTOK / 2;                        // tokens of x per CTA
  static constexpr int kXAtomBytes = kHalf * 128;               // kHalf rows x 128 B (64 inputs)
  static constexpr int kXBytes = 2 * kXAtomBytes;
  static constexpr int kStageBytes = kXBytes + 4 * kPairWTileBytes;
  static constexpr int kStages = NTOK == 256 ? 4 : 8;           // shared-memory ring (x + W)
  static constexpr int kDBufs = NTOK == 256 ? 1 : 2;            // accumulators
  static constexpr int kAColBase = kDBufs * NTOK;               // A stages after the accumulator(s)
  static constexpr int kEpiOffset = kStages * kStageBytes;
  static constexpr int kBarOffset = kEpiOffset + 2 * kPairEpiBufBytes;
  static_assert(kBarOffset + 512 + 1024 <= kPairSmemBytes, "pair kernel shared memory");
  static_assert(kPairSmemBytes <= 232448, "fits the 227 KB opt-in shared memory");
  static_assert(kAColBase + kPairAStages * kPairACols <= 512, "tensor memory budget");
};

struct PairParams {
  const void* bias;    // [4*N_g] or null
  void* y;             // [M, ld_y]
  int64_t ld_y;
  int M, N_g, K_g;
  int stages;          // K stages per tile: ceil(K_g / 32)
  int nb_tiles;        // tiles along the outputs: ceil(4*N_g / 256)
  int tiles;           // nb_tiles * ceil(M / NTOK)
  PeerOut peers;       // column-partitioned layer: every output also stored to these
};

// ---------------------------------------------------------------------------
// 2-SM tcgen05 helpers (inline PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D(tmem, both CTAs) (+)= A(tmem, both CTAs) * B(smem desc, both CTAs)^T, kind::f16.
__device__ __forceinline__ void umma_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrive once on the mbarrier at this shared-memory offset in every CTA of
// cta_mask when all UMMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(smem_u32(bar)), "h"(cta_mask) : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns per thread (warp-collective).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bounded mbarrier wait of this kernel.  The barrier may be completed from
// the other CTA of the pair (a remote arrive or a multicast UMMA commit); the
// default (CTA-scope) acquire of try_wait is used, as with the remote arrive
// below: the data a phase announces is either written by TMA or by
// tcgen05.st that the arriving thread has waited for, or read by UMMAs that
// the commit reports complete.
__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
  return mbar_wait(bar, parity, limit_ns);
}

// Arrive on the mbarrier at this shared-memory offset in CTA `cta` of the
// cluster (default semantics: release at CTA scope; a cluster-scope release
// here measured about 600 ns per arrive, serialising the builder warps).
__device__ __forceinline__ void mbar_arrive_cta(uint64_t* bar, uint32_t cta) {
  const uint32_t remote = map_peer_smem(smem_u32(bar), cta);
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

// UMMA shared-memory descriptor of a K-major operand tile written by TMA with
// 128-byte swizzling: 128-byte rows, 8-row groups of 1024 bytes (stride
// byte offset), leading byte offset unused, version 1, layout code 2.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= 1ull << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// 32 lanes x 32 bit, 32 consecutive columns per thread (warp-collective load).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Two fp32 values -> two 16-bit values in one word (low half = a).
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// PACKED: the weights come from the interleaved buffer wq[o][i][p] (the
// packed weight cache): a stage's W tile is two 32-row x 64-element boxes
// (16 input quaternions each, 128-byte swizzle) loaded through map_wr, and
// every builder lane reads all four components of an input quaternion from
// one 8-byte piece of its row -- no shuffles between lanes.
template <typename T, bool PEERS, int NTOK, bool PACKED = false>
__global__ void __launch_bounds__(kPairThreads, 1)
qlin_pair_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_wr,
                 const __grid_constant__ CUtensorMap map_wi, const __grid_constant__ CUtensorMap map_wj,
                 const __grid_constant__ CUtensorMap map_wk, const PairParams prm) {
  using Cfg = PairCfg<NTOK>;
  constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdesc = make_idesc_f16(256, NTOK, kFmt, false);
  constexpr int S = Cfg::kStages, SA = kPairAStages, NB = Cfg::kDBufs;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);  // [S] x and W of this CTA landed
  uint64_t* empty = full + S;     // [S] the UMMAs of the stage completed (both CTAs)
  uint64_t* afull = empty + S;    // [SA] even CTA: both CTAs' builders wrote the A stage
  uint64_t* aempty = afull + SA;  // [SA] the UMMAs reading the A stage completed (both CTAs)
  uint64_t* dfull = aempty + SA;  // [NB]
  uint64_t* dempty = dfull + NB;  // [NB], even CTA: both CTAs' epilogues drained the accumulator
  uint64_t* drain = dempty + NB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued = const_cast<int*>(abort_flag) + 1;  // producer: ring stages issued

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();     // 0: issues the UMMAs
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int my_tiles = pair < prm.tiles ? (prm.tiles - 1 - pair) / pairs + 1 : 0;
  const int nk = prm.stages;
  const int total = my_tiles * nk;  // ring items of this pair

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&afull[s], 8);
      mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&dfull[b], 1);
      mbar_init(&dempty[b], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *issued = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_wr);
    if (!PACKED) {
      tma_prefetch_desc(&map_wi);
      tma_prefetch_desc(&map_wj);
      tma_prefetch_desc(&map_wk);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised, tensor memory allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Everything below reads what earlier kernels of the stream wrote (x, W,
  // bias) or writes what they may read (y).
  pdl_wait_prior();

  auto tile_coords = [&](int t, int& n0, int& m0) {
    const int nb = t % prm.nb_tiles, tb = t / prm.nb_tiles;
    n0 = nb * 256 + (int)cta * kPairRows;  // this CTA's first real output
    m0 = tb * NTOK;                        // the pair's first token
  };

  if (warp == 0) {
    // ---------------- TMA producer: this CTA's x half-tile and W tiles ----------------
    if (lane == 0) {
      const CUtensorMap* wmap[4] = {&map_wr, &map_wi, &map_wj, &map_wk};
      int g = 0;
      for (int j = 0; j < my_tiles && !*abort_flag; ++j) {
        int n0, m0;
        tile_coords(pair + j * pairs, n0, m0);
        const int mrow = m0 + (int)cta * Cfg::kHalf;
        for (int k = 0; k < nk; ++k, ++g) {
          const int s = g % S, n = g / S;
          if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* dst = smem + s * Cfg::kStageBytes;
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          tma_load_2d(dst, &map_x, &full[s], k * kPairStageK, mrow);
          tma_load_2d(dst + Cfg::kXAtomBytes, &map_x, &full[s], k * kPairStageK + 64, mrow);
          if constexpr (PACKED) {
            // quaternions 32k .. 32k+15 and 32k+16 .. 32k+31 of rows n0/4 .. +31
#pragma unroll
            for (int h = 0; h < 2; ++h)
              tma_load_2d(dst + Cfg::kXBytes + h * 2 * kPairWTileBytes, &map_wr, &full[s],
                          k * kPairStageK + 64 * h, n0 / 4);
          } else {
#pragma unroll
            for (int p = 0; p < 4; ++p)
              tma_load_2d(dst + Cfg::kXBytes + p * kPairWTileBytes, wmap[p], &full[s], k * (kPairStageK / 4),
                          n0 / 4);
          }
          *issued = g + 1;
        }
        if (*abort_flag) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && cta == 0) {
      // ---------------- UMMA issuer (even CTA) ----------------
      bool ok = true;
      int g = 0;
      for (int j = 0; j < my_tiles && ok; ++j) {
        const int b = j % NB, u = j / NB;
        if (u > 0 && !mbar_wait(&dempty[b], (u - 1) & 1)) ok = false;
        tc_fence_after();
        for (int k = 0; k < nk && ok; ++k, ++g) {
          const int s = g % S, sa = g % SA, na = g / SA;
          // both CTAs' builders arrive only after their own CTA's x and W of
          // this stage landed: this one wait covers the B operand too
          if (!mbar_wait(&afull[sa], na & 1) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc0 = smem_desc_sw128(smem + s * Cfg::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < kPairStageK / 16; ++kk) {
            // K16 step kk: B bytes 32 (kk % 4) into swizzle atom kk / 4; A columns 8 kk
            const uint64_t bdesc = bdesc0 + (uint64_t)((kk >> 2) * (Cfg::kXAtomBytes >> 4)) + 2 * (kk & 3);
            umma_pair_ts(tmem + b * NTOK, tmem + Cfg::kAColBase + sa * kPairACols + 8 * kk, bdesc, kIdesc,
                         (k > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[s], 0x3);
          umma_commit_pair(&aempty[sa], 0x3);
        }
        if (ok) umma_commit_pair(&dfull[b], 0x3);
      }
      if (!ok) *abort_flag = 1;
      // every UMMA issued above has completed before the teardown
      umma_commit_pair(drain, 0x1);
      mbar_wait(drain, 0, 50000000ull);
    }
  } else if (warp < 6) {
    // ---------------- builders: expanded weight rows into tensor memory ----------------
    // Lane l of builder warp w writes tensor-memory lane 32 q + l (q = w % 4):
    // output quaternion o = n0/4 + 8 q + l % 8, component a = l / 8.  It reads
    // W_a[o, stage's 32 inputs] from the stage's swizzled W tile and takes
    // W_{a^q'} (q' = 1..3) from lanes l ^ 8 q' (same o).
    const int quarter = warp & 3;
    const int a = lane >> 3;
    const int row = 8 * quarter + (lane & 7);  // row of the 32-row W tiles
    uint32_t sg01, sg23;  // sign bits of values q = 0..3 of an input quaternion: s(a, a^q)
    {
      auto neg = [&](int q) {
        const int p = a ^ q;
        return (a == 0 && p != 0) || (a == 1 && p == 3) || (a == 2 && p == 1) || (a == 3 && p == 2);
      };
      sg01 = (neg(0) ? 0x8000u : 0u) | (neg(1) ? 0x80000000u : 0u);
      sg23 = (neg(2) ? 0x8000u : 0u) | (neg(3) ? 0x80000000u : 0u);
    }
    const uint32_t tm_lane = (uint32_t)(32 * quarter) << 16;
    for (int g = 0; g < total; ++g) {
      const int s = g % S, n = g / S, sa = g % SA, na = g / SA;
      bool ok = !*abort_flag && mbar_wait(&full[s], n & 1);
      if (ok && na > 0) ok = mbar_wait(&aempty[sa], (na - 1) & 1);
      if (!ok) *abort_flag = 1;
      if (!*abort_flag && PACKED) {
        // row `row` of the two packed boxes: 128 bytes each, 16-byte chunk c
        // (input quaternions 2c, 2c+1 of the box) at chunk c ^ (row & 7)
        const uint32_t col = tmem + tm_lane + Cfg::kAColBase + sa * kPairACols;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t wrow = smem_u32(smem + s * Cfg::kStageBytes + Cfg::kXBytes + h * 2 * kPairWTileBytes + row * 128);
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t q[4];
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3])
                         : "r"(wrow + ((c ^ (row & 7)) << 4))
                         : "memory");
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              // quaternion 2c+e: lo = (W_0, W_1), hi = (W_2, W_3); this row wants
              // (W_a, W_{a^1}) and (W_{a^2}, W_{a^3}), signed
              uint32_t lo = q[2 * e], hi = q[2 * e + 1];
              if (a & 2) {
                const uint32_t t = lo;
                lo = hi;
                hi = t;
              }
              if (a & 1) {
                lo = __byte_perm(lo, lo, 0x1032);
                hi = __byte_perm(hi, hi, 0x1032);
              }
              r[4 * c + 2 * e] = lo ^ sg01;
              r[4 * c + 2 * e + 1] = hi ^ sg23;
            }
          }
          tmem_st32(col + 32 * h, r);
        }
        tmem_st_wait();
      } else if (!*abort_flag) {
        // W_a[o, 32 inputs]: 64 bytes, chunk c at chunk c ^ ((row >> 1) & 3) (64-byte swizzle)
        const uint32_t wrow =
            smem_u32(smem + s * Cfg::kStageBytes + Cfg::kXBytes + a * kPairWTileBytes + row * 64);
        uint32_t w0[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t addr = wrow + ((c ^ ((row >> 1) & 3)) << 4);
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(w0[4 * c]), "=r"(w0[4 * c + 1]), "=r"(w0[4 * c + 2]), "=r"(w0[4 * c + 3])
                       : "r"(addr)
                       : "memory");
        }
        const uint32_t col = tmem + tm_lane + Cfg::kAColBase + sa * kPairACols;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          // input quaternions 16 h .. 16 h + 15: words 8 h .. 8 h + 7
          uint32_t r[32];
#pragma unroll
          for (int e8 = 0; e8 < 8; ++e8) {
            const int e = 8 * h + e8;
            const uint32_t v0 = w0[e];
            const uint32_t v1 = __shfl_xor_sync(0xffffffffu, v0, 8);
            const uint32_t v2 = __shfl_xor_sync(0xffffffffu, v0, 16);
            const uint32_t v3 = __shfl_xor_sync(0xffffffffu, v0, 24);
            // word e holds input quaternions 2e (low half) and 2e + 1 (high half)
            r[4 * e8 + 0] = __byte_perm(v0, v1, 0x5410) ^ sg01;
            r[4 * e8 + 1] = __byte_perm(v2, v3, 0x5410) ^ sg23;
            r[4 * e8 + 2] = __byte_perm(v0, v1, 0x7632) ^ sg01;
            r[4 * e8 + 3] = __byte_perm(v2, v3, 0x7632) ^ sg23;
          }
          tmem_st32(col + 32 * h, r);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(&afull[sa], 0);
    }
  } else {
    // ---------------- epilogue ----------------
    // Drain the accumulator into registers (bias added, rounded, two tokens
    // per word), release it to the UMMA issuer, then store through a
    // shared-memory transpose: 16 tokens x 128 outputs per group, 16 bytes per
    // thread and store.
    const int quarter = warp & 3;
    const int et = threadIdx.x - 192;  // 0..127
    const int n_local = 32 * quarter + 4 * (lane & 7) + (lane >> 3);
    T* __restrict__ y = reinterpret_cast<T*>(prm.y);
    const T* __restrict__ bias = reinterpret_cast<const T*>(prm.bias);
    for (int j = 0; j < my_tiles; ++j) {
      const int b = j % NB, u = j / NB;
      int n0, m0;
      tile_coords(pair + j * pairs, n0, m0);
      const bool got = !*abort_flag && mbar_wait(&dfull[b], u & 1);
      if (!got) *abort_flag = 1;
      tc_fence_after();
      const int n = n0 + n_local;
      const float bv = (bias && n < 4 * prm.N_g) ? to_f32(bias[n]) : 0.f;
      uint32_t packed[NTOK / 2];
#pragma unroll
      for (int c = 0; c < NTOK / 32; ++c) {
        uint32_t v[32];
        if (got) {
          __syncwarp();
          tmem_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + b * NTOK + 32 * c, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) v[t] = 0u;
        }
#pragma unroll
        for (int t = 0; t < 16; ++t)
          packed[16 * c + t] = pack2<T>(__uint_as_float(v[2 * t]) + bv, __uint_as_float(v[2 * t + 1]) + bv);
      }
      // this warp has read its lanes of the accumulator: the even CTA may reuse it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(&dempty[b], 0);
#pragma unroll
      for (int grp = 0; grp < NTOK / kPairEpiTokens; ++grp) {
        T* stage = reinterpret_cast<T*>(smem + Cfg::kEpiOffset + (grp & 1) * kPairEpiBufBytes);
        unsigned short* st16 = reinterpret_cast<unsigned short*>(stage);
#pragma unroll
        for (int t2 = 0; t2 < kPairEpiTokens / 2; ++t2) {
          const uint32_t wv = packed[(kPairEpiTokens / 2) * grp + t2];
          st16[(2 * t2) * kPairRows + n_local] = (unsigned short)(wv & 0xffffu);
          st16[(2 * t2 + 1) * kPairRows + n_local] = (unsigned short)(wv >> 16);
        }
        asm volatile("bar.sync %0, %1;" ::"n"(kPairEpiBar), "n"(128) : "memory");
        if (got) {
          // 16 tokens x 128 outputs = 256 pieces of 16 bytes, two per thread
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = et + 128 * h, t = c >> 4, cc = c & 15;
            const int m = m0 + kPairEpiTokens * grp + t, nn = n0 + 8 * cc;
            if (m < prm.M && nn < 4 * prm.N_g) {
              const uint4 v = *reinterpret_cast<const uint4*>(stage + t * kPairRows + 8 * cc);
              const int64_t off = (int64_t)m * prm.ld_y + nn;
              if (PEERS && prm.peers.mc) {
                multimem_st16(reinterpret_cast<T*>(prm.peers.mc) + off, v);
              } else {
                *reinterpret_cast<uint4*>(y + off) = v;
                if constexpr (PEERS) {
                  for (int pp = 0; pp < prm.peers.n; ++pp)
                    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(prm.peers.y[pp]) + off) = v;
                }
              }
            }
          }
        }
      }
    }
    if (PEERS) fence_sys();
  }

  // ---------------- teardown ----------------
  __syncwarp();
  if (threadIdx.x == 0 && *abort_flag) {
    // let issued TMA loads land before the shared memory goes away
    const int g1 = *issued;
    for (int g = g1 - S > 0 ? g1 - S : 0; g < g1; ++g) mbar_wait(&full[g % S], (g / S) & 1, 50000000ull);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while the other may still use its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace qlin
