// Tensor-core quaternion linear forward for sm_100a (TMA + tcgen05 + TMEM).
//
// Decomposition.  With component planes X_q[m, i] = x[m, 4i+q] the
// Hamilton-product layer is sixteen real products
//
//     Y_a[m, o] = sum_p s(a,p) * sum_i W_p[o, i] * X_{p^a}[m, i]
//
// (a = output component, p = weight component, q = p XOR a is the input
// component it pairs with, s(a,p) = +-1 is the sign of the 4x4 block matrix
// of reference quaternion/packing.py:18-21).  The A operand of every UMMA is
// a W_p tile exactly as TMA loads it from the caller's weight tensor, so each
// weight byte crosses HBM once per tile -- a quarter of a dense layer's
// traffic -- and the 4x real matrix is never formed anywhere.  The sign and
// component swap are applied on the activation side, in one of two ways:
//
//  * planes (M > 64): the prologue writes X_q planes to the workspace, TMA
//    loads them, and each (a, p) term is one UMMA (N = tokens) whose sign is
//    the instruction descriptor's negate-A bit -- 16 UMMAs per K step into
//    four TMEM accumulators;
//  * stacked (M <= 64): two builder warps read x directly and write, per
//    weight component p, the operand Xhat_p whose rows are (a, token) and
//    hold s(a,p) * X_{p^a}; one UMMA per p (N = 4 * tokens) then produces all
//    four output components at once -- 4 UMMAs per K step, each reading its
//    weight tile from shared memory once.
//
// In both modes accumulator column a * N_TOK + token holds Y_a, so the
// epilogue is shared.  CTA tile: 128 output quaternions (UMMA M = 128, one
// TMEM lane each) x N_TOK tokens.  K is walked in chunks of 32 input
// quaternions (64-byte rows, 64-byte TMA/UMMA swizzle).  With few tiles
// (decode) the chunks of one tile are split over several CTAs so that every
// SM streams weights; their fp32 partials of the real tokens go to the
// workspace and are summed by a small dependent kernel or, for at most four
// tokens on a zero-filled workspace, by the last CTA of the tile to finish
// (arrival counter).  LoRA: the scaled down
// projection t (prologue kernel) is the B operand of four extra UMMAs per 32
// ranks whose A operands are the [o, a]-strided rows of LoRA B, accumulated
// before the single rounding.
//
// Stream order: every kernel of this path is launched as a programmatic
// dependent of the previous kernel of the stream.  Its set-up (barriers,
// TMEM, descriptor prefetch) overlaps that kernel's tail, and it waits
// (griddepcontrol.wait) before it reads or writes memory -- except that with
// static weights (the caller's promise that earlier work does not write the
// weights) the first weight tiles are requested before the wait, and that
// after this call's prologue (which lets the main kernel launch only once it
// has itself waited for all earlier work) the main kernel streams weights and
// builds x operands while the prologue runs, waiting only before it loads
// the prologue's outputs.
//
// Roles (128 threads): thread 0 issues TMA, warp 1 owns TMEM and its lane 0
// issues UMMA, warps 2-3 build Xhat (stacked mode), all four warps run the
// epilogue (warp w reads TMEM lanes 32w..32w+31).  Every mbarrier wait is
// bounded (qlin_common.cuh); on a timeout the kernel records
// QLIN_ERR_TIMEOUT, skips the remaining work and still meets every barrier.
#pragma once

#include <type_traits>

#include "qlin_common.cuh"

namespace qlin {

constexpr int kTcBlockO = 128;   // output quaternions per CTA tile (UMMA M)
constexpr int kTcChunk = 32;     // input quaternions per K chunk (64-byte rows)
constexpr int kTcThreads = 128;      // TMA, UMMA, two builder warps; all four run the epilogue
constexpr int kTcLoraThreads = 64;   // CUDA-core LoRA: two more warps for the down projection
constexpr int kTcMaxThreads = kTcThreads + kTcLoraThreads;
constexpr int kTcEpiBar = 2;         // named barrier of the four epilogue warps
constexpr int kTcLoraBar = 3;        // named barrier of the two LoRA warps
constexpr int kTcWTileBytes = kTcBlockO * kTcChunk * 2;  // 8 KB
constexpr int kTcMaxSplit = 16;  // largest K split of one output tile
constexpr int kTcBuilderBar = 1; // named barrier of the two builder warps
constexpr int kTcLoraInRank = 32; // largest LoRA rank whose down projection runs in the main kernel
constexpr int kTcLoraSimtTokens = 4;  // largest M of the CUDA-core in-kernel down projection
constexpr int kTcLoraSliceBox = 256;  // elements per row of one lora_a slice load (CUDA-core mode)
constexpr int kTcLoraSliceMax = 512;  // elements of lora_a rows one split covers (4 chunks)
// LoRA down projection t = lora_scale * x A^T of the tensor-core kernel:
enum { kLoraPrologue = 0,  // none, or t from the prologue kernel (TMA-loaded)
       kLoraTc = 1,        // per split, on the tensor cores (extra UMMA per K step)
       kLoraSimt = 2 };    // per split, on the builder warps' CUDA cores
constexpr int kTcTLane = 64;      // TMEM lane of token 0 in the in-kernel LoRA accumulator

__host__ __device__ constexpr int tmem_cols_for(int n) {
  return n <= 32 ? 32 : (n <= 64 ? 64 : (n <= 128 ? 128 : (n <= 256 ? 256 : 512)));
}

// Cluster K split (decode, at most kTcClusterTokens tokens): every split of
// a tile is one CTA of a cluster of C CTAs (C = the split, at most
// kTcClusterMax; above 8 the non-portable cluster size).  A reduce-scatter
// through distributed shared memory: CTA r owns the tile's tokens
// [r * per, (r + 1) * per), per = ceil(tokens / C), receives every other
// split's fp32 partial of those tokens into its receive buffer
// [slot = sender (skipping itself) * per + owned token][128 rows] x float4
// (st.async, counted on its own mbarrier) and sums them in split order.
// (C - 1) * per stays within kTcClusterSlots for every C at up to 16 tokens.
constexpr int kTcClusterTokens = 16;
constexpr int kTcClusterMax = 16;
constexpr int kTcClusterSlots = 15;

template <int N_TOK, bool STACK, int LORA = kLoraPrologue, bool CLUSTER = false>
struct TcCfg {
  // Activation operand per weight component and stage: stacked [4*N_TOK rows]
  // or one plane [N_TOK rows], 64 bytes per row either way.
  static constexpr int kXTileBytes = (STACK ? 4 : 1) * N_TOK * kTcChunk * 2;
  // Stacked tiles: the chunk's raw x rows (4 sub-tiles of 32 elements x N_TOK
  // rows, 64-byte swizzle), brought by TMA and read by the builder warps
  // (and, in the tensor-core LoRA mode, the down projection's A operand);
  // there also the matching 32-element columns of lora_a (4 sub-tiles x
  // kTcLoraInRank rows).
  static constexpr int kRawXBytes = STACK ? 4 * N_TOK * 64 : 0;
  static constexpr int kLoraABytes = LORA == kLoraTc ? 4 * kTcLoraInRank * 64 : 0;
  static constexpr int kStageBytes = 4 * kTcWTileBytes + 4 * kXTileBytes + kRawXBytes + kLoraABytes;
  // CUDA-core LoRA: the split's lora_a slice [32 rows][<= 512 elements],
  // loaded once, ahead of the weights, as row pieces of kTcLoraSliceBox
  static constexpr int kSliceBytes = LORA == kLoraSimt ? kTcLoraInRank * kTcLoraSliceMax * 2 : 0;
  // Cluster K split: the receive buffer of the reduce-scatter aliases the
  // start of the stage ring (used only once every CTA of the cluster is past
  // its main loop), so it costs no stage.
  static constexpr int kRecvBytes = CLUSTER ? kTcClusterSlots * kTcBlockO * 16 : 0;
  static constexpr int kFit = (220 * 1024 - kSliceBytes) / kStageBytes;
  static constexpr int kStages = kFit > 6 ? 6 : (kFit < 2 ? 2 : kFit);
  static constexpr int kSliceOffset = kStages * kStageBytes;
  static constexpr int kRecvOffset = 0;
  // ... followed by the send buffer: this CTA's partials of every token,
  // [token][128 rows] x float4, from which one bulk copy per peer sends the
  // tokens that peer owns.
  static constexpr int kSendOffset = kRecvBytes;
  static constexpr int kSendBytes = CLUSTER ? kTcClusterTokens * kTcBlockO * 16 : 0;
  static_assert(kSendOffset + kSendBytes <= kStages * kStageBytes, "receive and send buffers inside the stage ring");
  // accumulators: 4*N_TOK columns of Y (+ kTcLoraInRank columns of t)
  static constexpr int kTmemCols = tmem_cols_for(4 * N_TOK + (LORA == kLoraTc ? kTcLoraInRank : 0));
  static constexpr int kBarOffset = kSliceOffset + kSliceBytes;
  static constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // + barriers + alignment slack
  static_assert(N_TOK == 16 || N_TOK == 32 || N_TOK == 64 || N_TOK == 128, "UMMA N");
  static_assert(!STACK || N_TOK <= 64, "stacked operand has 4*N_TOK <= 256 rows");
  static_assert(LORA != kLoraTc || (STACK && N_TOK <= 32), "tensor-core LoRA: stacked, tokens in lanes 64..95");
  static_assert(LORA != kLoraSimt || (STACK && N_TOK == 16), "CUDA-core LoRA: stacked, at most 4 tokens");
  static_assert(!CLUSTER || (STACK && N_TOK == 16), "cluster K split: decode tiles");
  // The LoRA down projection's A operand (128 rows from kTcTLane rows before
  // a raw x sub-tile) stays inside the stage: 4 KB of x operands before the
  // raw rows, at least 4 KB (raw rows + lora_a) after the last sub-tile.
  static_assert(LORA != kLoraTc || (4 * kTcWTileBytes + 4 * kXTileBytes >= kTcTLane * 64 &&
                             kRawXBytes / 4 + kLoraABytes >= (128 - kTcTLane) * 64),
                "LoRA A-operand window inside the stage");
  static_assert(kStageBytes % 1024 == 0, "stages keep 1024-byte alignment");
  static_assert(kSmemBytes <= 232448, "fits the 227 KB opt-in shared memory");
};

// neg(a, p): sign of W_p in output component a (rows of packing.py:18-21).
__host__ __device__ constexpr bool quat_neg(int a, int p) {
  return (a == 0 && p != 0) || (a == 1 && p == 3) || (a == 2 && p == 1) || (a == 3 && p == 2);
}

struct TcParams {
  const void* x;       // [M, ld_x] (stacked mode reads it directly)
  int64_t ld_x;
  const void* bias;    // [4*N_g] or null
  void* y;             // [M, ld_y]
  int64_t ld_y;
  int M, N_g, K_g;
  int num_chunks;      // ceil(K_g / 32)
  int lora_chunks;     // ceil(rank / 32), 0 without LoRA
  int split_k;         // CTAs sharing one output tile along K (1 = no split)
  float4* partials;    // split_k > 1: [split][t_blocks][o_blocks][N_TOK][128] fp32 x4
  unsigned* counters;  // fused reduction: one arrival counter per output tile, zero between calls
  int fuse_reduce;     // split_k > 1: the last CTA of a tile to arrive sums the partials
  int static_weights;  // weights/bias/LoRA B are not written by earlier work on the stream
  int after_prologue;  // launched right after this call's prologue kernel (see below)
  int no_cluster;      // host-side choice only: QLIN_FLAG_NO_CLUSTER
  int sub3d;           // stacked tiles: map_x (and the tensor-core mode's map_la) are 3-D views
                       // [sub-tile][row][32 elements], one box per chunk instead of four
  int rank;            // LoRA rank (in-kernel LoRA: ranks >= rank are zero)
  float lora_scale;    // in-kernel LoRA: t = lora_scale * x A^T
  const void* lora_a;  // CUDA-core in-kernel LoRA: A [rank, ld_a]
  int64_t ld_a;
  PeerOut peers;       // column-partitioned layer: every output also stored to these
};

__device__ __forceinline__ void builder_bar_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kTcBuilderBar), "n"(64) : "memory");
}
__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kTcEpiBar), "n"(kTcThreads) : "memory");
}
__device__ __forceinline__ void lora_bar_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kTcLoraBar), "n"(kTcLoraThreads) : "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Arrive (default semantics) on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr) : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// fence.acq_rel.gpu, then a relaxed gpu-scope atomic add; returns the old value.
__device__ __forceinline__ unsigned atomic_add_release_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("fence.acq_rel.gpu;\n\tatom.relaxed.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Cluster K split, owner side: acc += the C splits' partials of one token in
// split order (split ks from mine_addr, split sp != ks from receive slot
// sp - (sp > ks), slot_bytes apart from recv_addr); MAXC >= C.  The loads are
// issued together, then summed.
template <int MAXC>
__device__ __forceinline__ void tc_cluster_sum(float4& acc, int C, int ks, uint32_t mine_addr,
                                               uint32_t recv_addr, uint32_t slot_bytes) {
  uint32_t r[MAXC][4];
#pragma unroll
  for (int sp = 0; sp < MAXC; ++sp) {
    const uint32_t addr = sp == ks ? mine_addr : recv_addr + (uint32_t)(sp - (sp > ks ? 1 : 0)) * slot_bytes;
    if (sp < C) ld_shared_v4(addr, r[sp][0], r[sp][1], r[sp][2], r[sp][3]);
  }
#pragma unroll
  for (int sp = 0; sp < MAXC; ++sp) {
    if (sp < C) {
      acc.x += __uint_as_float(r[sp][0]);
      acc.y += __uint_as_float(r[sp][1]);
      acc.z += __uint_as_float(r[sp][2]);
      acc.w += __uint_as_float(r[sp][3]);
    }
  }
}

template <typename T, int N_TOK, bool STACK, int LORA, bool PEERS, bool CLUSTER = false>
__global__ void __launch_bounds__(kTcMaxThreads, 1)
qlin_tc_kernel(const __grid_constant__ CUtensorMap map_wr, const __grid_constant__ CUtensorMap map_wi,
               const __grid_constant__ CUtensorMap map_wj, const __grid_constant__ CUtensorMap map_wk,
               const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_lb,
               const __grid_constant__ CUtensorMap map_t, const __grid_constant__ CUtensorMap map_la,
               const TcParams prm) {
  using Cfg = TcCfg<N_TOK, STACK, LORA, CLUSTER>;
  constexpr int S = Cfg::kStages;
  // Activation operands built in shared memory by the builder warps
  // (stacked tiles) or TMA-loaded from the prologue's planar copy of x
  // (plane tiles; building those in the kernel measured 1.5x slower for
  // 128-token tiles: two builder warps cannot feed the tensor cores).
  constexpr bool kBuilt = STACK;
  constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescPos = make_idesc_f16(128, N_TOK, kFmt, false);
  constexpr uint32_t kIdescNeg = make_idesc_f16(128, N_TOK, kFmt, true);
  constexpr uint32_t kIdescStack = make_idesc_f16(128, STACK ? 4 * N_TOK : N_TOK, kFmt, false);
  constexpr uint32_t kIdescLoraDown = make_idesc_f16(128, kTcLoraInRank, kFmt, false);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* t_full = acc_full + 1;  // LoRA: down projection complete (tensor cores) / lora_a slice loaded (CUDA cores)
  uint64_t* red_full = t_full + 1;  // fused K-split reduction: all partials are in shared memory
  uint64_t* gather = red_full + 1;  // cluster K split (leader): every peer's partial has arrived
  uint64_t* xfull = gather + 1;     // stacked tiles: the stage's raw x rows have landed
  uint64_t* peers_free = xfull + S; // cluster K split: every other CTA is past its main loop
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(peers_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_count = const_cast<int*>(abort_flag) + 1;
  int* consumed_count = issued_count + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = blockIdx.y * kTcBlockO;
  const int t0 = blockIdx.z * N_TOK;
  const int ks = blockIdx.x;  // K split index
  const int c_begin = (int)((int64_t)ks * prm.num_chunks / prm.split_k);
  const int c_end = (int)((int64_t)(ks + 1) * prm.num_chunks / prm.split_k);
  const int my_main = c_end - c_begin;
  // With the down projection in this kernel every split applies the LoRA up
  // projection to its own partial t (a linear term, summed with the split);
  // otherwise the last split applies it to the prologue's full t.
  const int my_lora = (LORA != kLoraPrologue || ks == prm.split_k - 1) ? prm.lora_chunks : 0;
  const int total = my_main + my_lora;
  const int m_tile = (prm.M - t0) < N_TOK ? (prm.M - t0) : N_TOK;  // real tokens in the tile

  // The next kernel of the stream may launch now: every kernel of this path
  // waits (griddepcontrol.wait) for its predecessor to complete before it
  // reads or writes memory the predecessor may use.
  pdl_launch_dependents();
  // After a prologue, this grid only launches once every prologue CTA has
  // passed its own griddepcontrol.wait, i.e. once all work queued before
  // this call has completed.  Weights, bias, x and y are then safe to touch
  // at once; only the prologue's outputs (x planes, LoRA t) are waited for,
  // by the TMA producer, before its first load of them.
  const bool early = prm.static_weights || prm.after_prologue;

  auto w_tile = [&](int s, int p) { return smem + s * Cfg::kStageBytes + p * kTcWTileBytes; };
  auto x_tile = [&](int s, int q) {
    return smem + s * Cfg::kStageBytes + 4 * kTcWTileBytes + q * Cfg::kXTileBytes;
  };
  auto raw_tile = [&](int s, int j) {  // raw x rows, elements 32j..32j+31 of the chunk
    return smem + s * Cfg::kStageBytes + 4 * kTcWTileBytes + 4 * Cfg::kXTileBytes + j * N_TOK * 64;
  };
  auto la_tile = [&](int s, int j) {  // lora_a rows, the same 32 elements
    return smem + s * Cfg::kStageBytes + 4 * kTcWTileBytes + 4 * Cfg::kXTileBytes + Cfg::kRawXBytes +
           j * kTcLoraInRank * 64;
  };
  const CUtensorMap* wmap[4] = {&map_wr, &map_wi, &map_wj, &map_wk};
  const int pre = total < S ? total : S;
  // Stacked tiles: the raw x rows of main-loop stage it (after the
  // dependency wait: x may come from the previous kernel of the stream).
  auto issue_raw_x = [&](int it) {
    const int s = it % S, k = (c_begin + it) * kTcChunk;
    mbar_arrive_expect_tx(&xfull[s], (uint32_t)Cfg::kRawXBytes);
    if (prm.sub3d) {
      tma_load_3d(raw_tile(s, 0), &map_x, &xfull[s], 0, t0, k / 8);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) tma_load_2d(raw_tile(s, j), &map_x, &xfull[s], 4 * k + 32 * j, t0);
    }
  };
  // lora_a columns of the chunk at input quaternion k (tensor-core LoRA mode)
  auto issue_lora_a = [&](int s, int k) {
    if (prm.sub3d) {
      tma_load_3d(la_tile(s, 0), &map_la, &full[s], 0, 0, k / 8);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) tma_load_2d(la_tile(s, j), &map_la, &full[s], 4 * k + 32 * j, 0);
    }
  };
  // Weight (and LoRA B) tiles of the first stages; in the CUDA-core LoRA mode
  // preceded by this split's lora_a slice, so that it arrives first.
  auto issue_pre_weights = [&]() {
    if (LORA == kLoraSimt) {
      const int pieces = (4 * kTcChunk * my_main + kTcLoraSliceBox - 1) / kTcLoraSliceBox;
      mbar_arrive_expect_tx(t_full, pieces * kTcLoraInRank * kTcLoraSliceBox * 2);
      for (int j = 0; j < pieces; ++j)
        tma_load_2d(smem + Cfg::kSliceOffset + j * kTcLoraInRank * kTcLoraSliceBox * 2, &map_la, t_full,
                    4 * kTcChunk * c_begin + kTcLoraSliceBox * j, 0);
    }
    for (int it = 0; it < pre; ++it) {
      if (it < my_main) {
        const int k = (c_begin + it) * kTcChunk;
        mbar_arrive_expect_tx(&full[it], 4 * kTcWTileBytes + (kBuilt ? 0 : 4 * Cfg::kXTileBytes) +
                                             Cfg::kLoraABytes);
#pragma unroll
        for (int p = 0; p < 4; ++p) tma_load_2d(w_tile(it, p), wmap[p], &full[it], k, o0);
        if (LORA == kLoraTc) {
          issue_lora_a(it, k);
        }
      } else {
        const int r = (it - my_main) * kTcChunk;
        mbar_arrive_expect_tx(&full[it], 4 * kTcWTileBytes + (LORA != kLoraPrologue ? 0 : N_TOK * kTcChunk * 2));
#pragma unroll
        for (int a = 0; a < 4; ++a) tma_load_3d(w_tile(it, a), &map_lb, &full[it], r, a, o0);
      }
    }
  };
  // Bias of this thread's output row as raw bits; converted in the epilogue,
  // so the load latency hides under the main loop.  With a K split the bias
  // is added by the reduction kernel, or by the last CTA of the tile to
  // arrive when the reduction is fused.
  auto load_bias = [&](T (&raw)[4]) {
    const int ob = o0 + (int)threadIdx.x;
    const T* __restrict__ bp = reinterpret_cast<const T*>(prm.bias);
    const bool has = bp && (prm.split_k == 1 || prm.fuse_reduce || CLUSTER) && ob < prm.N_g &&
                     threadIdx.x < kTcBlockO;
#pragma unroll
    for (int a = 0; a < 4; ++a) raw[a] = has ? bp[4 * ob + a] : from_f32<T>(0.f);
  };

  // Set-up that touches no global memory, so it overlaps the tail of the
  // previous kernel of the stream.
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], kBuilt ? 2 : 1);  // producer (+ builders)
      mbar_init(&empty[s], 1);
      mbar_init(&xfull[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(t_full, 1);
    mbar_init(red_full, 1);
    mbar_init(gather, 1);
    mbar_init(peers_free, CLUSTER && prm.split_k > 1 ? prm.split_k - 1 : 1);
    // every owner arms its receive barrier before any peer can send (the
    // cluster barrier below orders this before every peer's epilogue)
    if (CLUSTER) {
      const int per = (m_tile + prm.split_k - 1) / prm.split_k;
      const int n_own = min(m_tile, (ks + 1) * per) - ks * per;
      if (n_own > 0) mbar_arrive_expect_tx(gather, (uint32_t)((prm.split_k - 1) * n_own * kTcBlockO * 16));
    }
    *abort_flag = 0;
    *issued_count = 0;
    *consumed_count = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_wr);
    tma_prefetch_desc(&map_wi);
    tma_prefetch_desc(&map_wj);
    tma_prefetch_desc(&map_wk);
    tma_prefetch_desc(&map_x);
    if (LORA != kLoraPrologue) tma_prefetch_desc(&map_la);
    // With static weights the caller guarantees that no earlier work on the
    // stream writes the weights, bias or LoRA A/B, so their first tiles are
    // requested before waiting for that work.
    if (early) issue_pre_weights();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  T bias_raw[4];
  if (early) load_bias(bias_raw);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (CLUSTER) cluster_sync_all();  // every CTA's barriers are initialised
  const uint32_t tmem_base = *tmem_slot;
  // Everything below may read what earlier kernels of the stream wrote (x,
  // the prologue's outputs, the workspace) or write what they read (y).
  // (the CUDA-core LoRA warps wait on their own, after their first loads)
  if (!prm.after_prologue && !(LORA == kLoraSimt && warp >= 4)) pdl_wait_prior();
  if (!early) load_bias(bias_raw);

  if (threadIdx.x == 0) {
    // ---------------- TMA producer ----------------
    if (!early) issue_pre_weights();
    if (kBuilt)
      for (int it = 0; it < pre && it < my_main; ++it) issue_raw_x(it);
    if (prm.after_prologue && (!kBuilt || my_lora > 0)) pdl_wait_prior();  // x planes / LoRA t
    for (int it = 0; it < pre; ++it) {
      if (it < my_main) {
        if (!kBuilt) {
          const int k = (c_begin + it) * kTcChunk;
#pragma unroll
          for (int q = 0; q < 4; ++q) tma_load_3d(x_tile(it, q), &map_x, &full[it], k, t0, q);
        }
      } else if (LORA == kLoraPrologue) {
        tma_load_2d(x_tile(it, 0), &map_t, &full[it], (it - my_main) * kTcChunk, t0);
      }
    }
    int it = pre;
    for (; it < total; ++it) {
      const int s = it % S, n = it / S;
      if (!mbar_wait(&empty[s], (n - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      if (it < my_main) {
        const int k = (c_begin + it) * kTcChunk;
        if (kBuilt) issue_raw_x(it);
        mbar_arrive_expect_tx(&full[s], 4 * kTcWTileBytes + (kBuilt ? 0 : 4 * Cfg::kXTileBytes) +
                                            Cfg::kLoraABytes);
#pragma unroll
        for (int p = 0; p < 4; ++p) tma_load_2d(w_tile(s, p), wmap[p], &full[s], k, o0);
        if (!kBuilt) {
#pragma unroll
          for (int q = 0; q < 4; ++q) tma_load_3d(x_tile(s, q), &map_x, &full[s], k, t0, q);
        }
        if (LORA == kLoraTc) {
          issue_lora_a(s, k);
        }
      } else {
        const int r = (it - my_main) * kTcChunk;
        mbar_arrive_expect_tx(&full[s], 4 * kTcWTileBytes + (LORA != kLoraPrologue ? 0 : N_TOK * kTcChunk * 2));
#pragma unroll
        for (int a = 0; a < 4; ++a) tma_load_3d(w_tile(s, a), &map_lb, &full[s], r, a, o0);
        if (LORA == kLoraPrologue) tma_load_2d(x_tile(s, 0), &map_t, &full[s], r, t0);
      }
    }
    *issued_count = it;
  } else if (threadIdx.x == 32) {
    // ---------------- UMMA issuer ----------------
    int it = 0;
    for (; it < total; ++it) {
      const int s = it % S, n = it / S;
      if (!mbar_wait(&full[s], n & 1)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      if (it < my_main) {
#pragma unroll
        for (int kk = 0; kk < kTcChunk / 16; ++kk) {
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint64_t adesc = smem_desc_sw64(w_tile(s, p)) + 2 * kk;
            const uint32_t accum = (it > 0 || kk > 0 || p > 0) ? 1u : 0u;
            if (STACK) {
              umma_f16(tmem_base, adesc, smem_desc_sw64(x_tile(s, p)) + 2 * kk, kIdescStack, accum);
            } else {
#pragma unroll
              for (int a = 0; a < 4; ++a)
                umma_f16(tmem_base + a * N_TOK, adesc, smem_desc_sw64(x_tile(s, p ^ a)) + 2 * kk,
                         quat_neg(a, p) ? kIdescNeg : kIdescPos, accum);
            }
          }
        }
        if (LORA == kLoraTc) {
          // t^T partial: D[lane kTcTLane + token][rank] += x[token, k] * A[rank, k]
          // over the chunk's four 32-element sub-tiles.  The A operand starts
          // kTcTLane rows before the raw rows; the other rows' lanes are never read.
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
              umma_f16(tmem_base + 4 * N_TOK, smem_desc_sw64(raw_tile(s, j) - kTcTLane * 64) + 2 * kk,
                       smem_desc_sw64(la_tile(s, j)) + 2 * kk, kIdescLoraDown,
                       (it > 0 || j > 0 || kk > 0) ? 1u : 0u);
        }
      } else {
#pragma unroll
        for (int kk = 0; kk < kTcChunk / 16; ++kk) {
          const uint64_t bdesc = smem_desc_sw64(x_tile(s, 0)) + 2 * kk;
#pragma unroll
          for (int a = 0; a < 4; ++a)
            umma_f16(tmem_base + a * N_TOK, smem_desc_sw64(w_tile(s, a)) + 2 * kk, bdesc, kIdescPos, 1u);
        }
      }
      umma_commit(&empty[s]);
      if (LORA == kLoraTc && it == my_main - 1) umma_commit(t_full);
    }
    *consumed_count = it;
    umma_commit(acc_full);  // fires once every UMMA issued above has completed
  } else if (kBuilt && (warp == 2 || warp == 3)) {
    // ---------------- Xhat builders (warps 2-3) ----------------
    // Xhat_p row (a*N_TOK + token), 16-byte chunk c (input groups 8c..8c+7
    // of the chunk) = s(a,p) * X_{p^a}: one work item moves 8 quaternions of
    // one token (64 bytes of x) into 16 swizzled 16-byte slots (64-byte
    // swizzle: chunk c of row r sits at chunk c ^ ((r >> 1) & 3)).  Every
    // builder runs every iteration (and meets every named barrier) even after
    // an abort, so no builder can be left waiting.
    const int bt = threadIdx.x - 64;
    bool t_seen = false;
    // With the CUDA-core LoRA the LoRA stages belong to warps 4-5.
    const int b_total = LORA == kLoraSimt ? my_main : total;
    for (int it = 0; it < b_total; ++it) {
      const int s = it % S, n = it / S;
      if (it >= S && !*abort_flag && !mbar_wait(&empty[s], (n - 1) & 1)) *abort_flag = 1;
      if (it < my_main && !*abort_flag) {
        // The stage's raw x rows arrive by TMA (64-byte swizzle: 16-byte
        // chunk c of row r at chunk c ^ ((r >> 1) & 3)); N_TOK*4 items of 64
        // bytes, kItems per builder.  (Loading x here from global memory put
        // one L2 round trip per stage on the builders' path: measured, it
        // held the decode kernel at one stage per microsecond per CTA.)
        if (!mbar_wait(&xfull[s], n & 1)) *abort_flag = 1;
        constexpr int kItems = N_TOK * 4 / 64;
#pragma unroll
        for (int k = 0; k < kItems; ++k) {
          const int item = bt + 64 * k;
          const int tok = item >> 2, gb = item & 3;
          const uint32_t rbase = smem_u32(raw_tile(s, gb)) + tok * 64;
          uint32_t w[16];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            ld_shared_v4(rbase + ((c ^ ((tok >> 1) & 3)) << 4), w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
          // plane q of the 8 quaternions: word j = (X_q[2j], X_q[2j+1])
          uint32_t pl[4][4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int j = 0; j < 4; ++j)
              pl[q][j] = __byte_perm(w[4 * j + (q >> 1)], w[4 * j + 2 + (q >> 1)], (q & 1) ? 0x7632 : 0x5410);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint32_t base = smem_u32(x_tile(s, p));
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int a = p ^ q;
              const uint32_t sg = quat_neg(a, p) ? 0x80008000u : 0u;
              const int row = a * N_TOK + tok;
              const uint32_t addr = base + row * 64 + ((gb ^ ((row >> 1) & 3)) << 4);
              st_shared_v4(addr, pl[q][0] ^ sg, pl[q][1] ^ sg, pl[q][2] ^ sg, pl[q][3] ^ sg);
            }
          }
        }
        fence_async_smem();
      } else if (LORA == kLoraTc && it >= my_main && !*abort_flag) {
        // LoRA up projection operand: t = lora_scale * (this split's t^T
        // partial), rounded once; warp 2 reads TMEM lanes 64..95 (tokens).
        if (!t_seen) {
          if (!mbar_wait(t_full, 0)) *abort_flag = 1;
          tc_fence_after();
          t_seen = true;
        }
        if (warp == 2) {
          float v0[16], v1[16];
          const uint32_t taddr = tmem_base + ((uint32_t)kTcTLane << 16) + 4 * N_TOK;
          __syncwarp();  // tcgen05.ld is warp-collective
          tmem_ld16(taddr, v0);
          tmem_ld16(taddr + 16, v1);
          tmem_ld_wait();
          const int tok = lane;
          if (tok < N_TOK && !*abort_flag) {
            const uint32_t tb = smem_u32(x_tile(s, 0)) + tok * 64;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int r = 8 * c + e;
                f[e] = r < prm.rank ? prm.lora_scale * (r < 16 ? v0[r] : v1[r - 16]) : 0.f;
              }
              const uint2 lo = pack4<T>(f[0], f[1], f[2], f[3]);
              const uint2 hi = pack4<T>(f[4], f[5], f[6], f[7]);
              st_shared_v4(tb + ((c ^ ((tok >> 1) & 3)) << 4), lo.x, lo.y, hi.x, hi.y);
            }
          }
          fence_async_smem();
        }
      }
      builder_bar_sync();
      if (bt == 0) mbar_arrive(&full[s]);
    }
  } else if (LORA == kLoraSimt && warp >= 4) {
    // ---------------- LoRA down projection (warps 4-5, CUDA cores) ----------------
    // Warp lw owns ranks 16lw..16lw+15; lane l takes elements 8l..8l+7
    // (+256j) of this split's slice: x from global memory (512 contiguous
    // bytes per warp load), lora_a from the shared slice the producer loaded
    // ahead of the weights (conflict-free 16-byte reads).  The per-lane
    // partial dot products are summed by a transposing butterfly after which
    // lane pair (2k, 2k+1) holds rank 16lw+k, for every token.
    const int lt = threadIdx.x - kTcThreads;
    const int lw = lt >> 5;
    const int r = 16 * lw + (lane >> 1), h = lane & 1;  // rank and row parity this lane writes
    const T* __restrict__ x = reinterpret_cast<const T*>(prm.x);
    const int E = 4 * kTcChunk * my_main;  // elements of this split, at most 512
    const int ebase = 4 * kTcChunk * c_begin;
    const int lim = 4 * prm.K_g;
    if (!prm.after_prologue) pdl_wait_prior();
    // x pieces of this lane (each token, each 256-element piece)
    uint4 xv[kTcLoraSimtTokens][2];
#pragma unroll
    for (int m = 0; m < kTcLoraSimtTokens; ++m)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int eo = 256 * j + 8 * lane, e = ebase + eo;
        xv[m][j] = (m < m_tile && eo < E && e < lim)
                       ? ld_cg_v4(x + (int64_t)(t0 + m) * prm.ld_x + e)
                       : make_uint4(0u, 0u, 0u, 0u);
      }
    // the lora_a slice: [piece j][rank][256 elements], rows past rank zero
    const bool a_ok = mbar_wait(t_full, 0);
    if (!a_ok) *abort_flag = 1;
    const uint4* slice = reinterpret_cast<const uint4*>(smem + Cfg::kSliceOffset);
    float tacc[kTcLoraSimtTokens];
#pragma unroll
    for (int m = 0; m < kTcLoraSimtTokens; ++m) {
      float vals[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) vals[k] = 0.f;
      if (m < m_tile && a_ok) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (256 * j < E) {
#pragma unroll
            for (int k = 0; k < 16; ++k)
              vals[k] += dot8<T>(slice[(j * kTcLoraInRank + 16 * lw + k) * (kTcLoraSliceBox / 8) + lane], xv[m][j]);
          }
        }
      }
      // butterfly over lane bits 4..1: keep the half of the values selected
      // by the lane bit, add the partner's other half
#pragma unroll
      for (int o = 16, n = 16; o >= 2; o >>= 1, n >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
          const float send = upper ? vals[i] : vals[i + n / 2];
          const float keep = upper ? vals[i + n / 2] : vals[i];
          vals[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      tacc[m] = vals[0] + __shfl_xor_sync(0xffffffffu, vals[0], 1);
    }
    for (int it = my_main; it < total; ++it) {
      const int s = it % S, n = it / S;
      if (it >= S && !*abort_flag && !mbar_wait(&empty[s], (n - 1) & 1)) *abort_flag = 1;
      if (!*abort_flag) {
        const uint32_t tb = smem_u32(x_tile(s, 0));
#pragma unroll
        for (int m = h; m < N_TOK; m += 2) {
          float v = 0.f;
#pragma unroll
          for (int mm = 0; mm < kTcLoraSimtTokens; ++mm)
            if (mm == m) v = tacc[mm];
          const T val = from_f32<T>((m < m_tile && r < prm.rank) ? prm.lora_scale * v : 0.f);
          const uint32_t addr = tb + m * 64 + (((r >> 3) ^ ((m >> 1) & 3)) << 4) + (r & 7) * 2;
          asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr),
                       "h"(*reinterpret_cast<const unsigned short*>(&val))
                       : "memory");
        }
        fence_async_smem();
      }
      lora_bar_sync();
      if (lt == 0) mbar_arrive(&full[s]);
    }
  }
  __syncwarp();

  // ---------------- epilogue ----------------
  // Warps 0-3 own the 128 TMEM lanes (one output row each); the LoRA warps
  // of the CUDA-core mode go straight to the teardown.
  if (warp < 4) {
    const bool acc_ok = mbar_wait(acc_full, 0);
    tc_fence_after();
    const bool ok = acc_ok && (*abort_flag == 0);
    const int o_local = warp * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(warp * 32) << 16);
    T* __restrict__ y = reinterpret_cast<T*>(prm.y);
    const int jn = (m_tile + 15) / 16;  // 16-token column groups holding real tokens

    if (prm.split_k == 1) {
      const int o = o0 + o_local;
      float b[4];
  #pragma unroll
      for (int a = 0; a < 4; ++a) b[a] = to_f32(bias_raw[a]);
  #pragma unroll 1
      for (int j = 0; j < jn; ++j) {
        float v[4][16];
  #pragma unroll
        for (int a = 0; a < 4; ++a) tmem_ld16(lane_addr + a * N_TOK + j * 16, v[a]);
        tmem_ld_wait();
        if (ok && o < prm.N_g) {
  #pragma unroll
          for (int t = 0; t < 16; ++t) {
            const int m = t0 + j * 16 + t;
            if (m < prm.M) {
              store_out<T, PEERS>(y, prm.peers, (int64_t)m * prm.ld_y + 4 * o,
                           pack4<T>(v[0][t] + b[0], v[1][t] + b[1], v[2][t] + b[2], v[3][t] + b[3]));
            }
          }
        }
      }
    } else if (CLUSTER) {
      // Cluster K split (reduce-scatter, see kTcClusterTokens): this CTA's
      // fp32 partials of the tokens other CTAs own go to their receive
      // buffers -- staged in this CTA's send buffer, then one bulk copy per
      // owner (shared::cta -> shared::cluster, counted on the owner's gather
      // barrier), sent even after an abort so every owner's count completes
      // -- and the owned tokens are summed over all splits in split order,
      // plus the bias.
      const int C = prm.split_k;
      const int per = (m_tile + C - 1) / C;
      const int own0 = ks * per;
      const int n_own = min(m_tile, own0 + per) - own0;
      float v[4][16];
#pragma unroll
      for (int a = 0; a < 4; ++a) tmem_ld16(lane_addr + a * N_TOK, v[a]);
      tmem_ld_wait();
      // The receive buffers alias the stage rings: tell every other CTA that
      // this one is past its main loop (its last UMMA has read its stages),
      // and send only once all of them are.  This CTA's own ring is free
      // once its accumulator is complete, so the send buffer is filled first.
      // Lane q of warp 0 handles peer q.  The code stays free of divisions
      // and data-dependent branches: with one warp per SM sub-partition
      // nothing hides their latency (a per-token owner test t / per cost
      // ~1.3 us per call here, the unconditional stores 0.35 us).
      const int q = lane;
      const bool peer = warp == 0 && q < C && q != ks;
      if (peer) mbar_arrive_remote(map_peer_smem(smem_u32(peers_free), (uint32_t)q));
      const uint32_t send = smem_u32(smem + Cfg::kSendOffset);
#pragma unroll
      for (int t = 0; t < kTcClusterTokens; ++t)  // every token; only the peers' ranges are sent
        st_shared_v4(send + (uint32_t)((t * kTcBlockO + o_local) * 16), __float_as_uint(v[0][t]),
                     __float_as_uint(v[1][t]), __float_as_uint(v[2][t]), __float_as_uint(v[3][t]));
      fence_async_smem();  // generic-proxy stores -> bulk copy reads
      epi_bar_sync();
      if (warp == 0) {
        if (!mbar_wait(peers_free, 0)) *abort_flag = 1;
        const int nq = min(m_tile, (q + 1) * per) - q * per;  // tokens owner q holds
        if (peer && nq > 0) {
          const int slot = (ks < q ? ks : ks - 1) * per;
          bulk_copy_to_peer(map_peer_smem(smem_u32(smem + Cfg::kRecvOffset), (uint32_t)q) +
                                (uint32_t)(slot * kTcBlockO * 16),
                            send + (uint32_t)(q * per * kTcBlockO * 16), (uint32_t)(nq * kTcBlockO * 16),
                            map_peer_smem(smem_u32(gather), (uint32_t)q));
        }
      }
      if (n_own > 0) {
        const bool got = mbar_wait(gather, 0);
        const int o = o0 + o_local;
        float b[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) b[a] = to_f32(bias_raw[a]);
        // Split sp's partial of owned token own0 + tl: this CTA's own from
        // the send buffer, the others from receive slot (sp - (sp > ks)) * per
        // + tl.  All loads first, then the sum in split order.
        const uint32_t mine_addr = send + (uint32_t)((own0 * kTcBlockO + o_local) * 16);
        const uint32_t recv_addr = smem_u32(smem + Cfg::kRecvOffset) + (uint32_t)(o_local * 16);
        const uint32_t slot_bytes = (uint32_t)(per * kTcBlockO * 16);
        for (int tl = 0; tl < n_own; ++tl) {
          const uint32_t tok_off = (uint32_t)(tl * kTcBlockO * 16);
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          if (C <= 8) {
            tc_cluster_sum<8>(acc, C, ks, mine_addr + tok_off, recv_addr + tok_off, slot_bytes);
          } else {
            tc_cluster_sum<kTcClusterMax>(acc, C, ks, mine_addr + tok_off, recv_addr + tok_off, slot_bytes);
          }
          if (ok && got && o < prm.N_g)
            store_out<T, PEERS>(y, prm.peers, (int64_t)(t0 + own0 + tl) * prm.ld_y + 4 * o,
                                pack4<T>(acc.x + b[0], acc.y + b[1], acc.z + b[2], acc.w + b[3]));
        }
      }
    } else {
      // K split: fp32 partials of the real tokens go to this CTA's slot of the
      // workspace as [token][row] float4 (a = 0..3).  They are summed with the
      // bias and rounded either by qlin_splitk_reduce_kernel or, for a few
      // tokens, here: the last CTA of the tile to arrive (arrival counter in the
      // workspace, reset to zero by that CTA) reads all slots in split order.
      const size_t slot_stride = (size_t)gridDim.z * gridDim.y * (N_TOK * kTcBlockO);
      const size_t tile_off = ((size_t)blockIdx.z * gridDim.y + blockIdx.y) * (N_TOK * kTcBlockO);
      float4* part = prm.partials + (size_t)ks * slot_stride + tile_off;
  #pragma unroll 1
      for (int j = 0; j < jn; ++j) {
        float v[4][16];
  #pragma unroll
        for (int a = 0; a < 4; ++a) tmem_ld16(lane_addr + a * N_TOK + j * 16, v[a]);
        tmem_ld_wait();
        if (ok) {
  #pragma unroll
          for (int t = 0; t < 16; ++t) {
            const int tok = j * 16 + t;
            if (tok < m_tile) part[tok * kTcBlockO + o_local] = make_float4(v[0][t], v[1][t], v[2][t], v[3][t]);
          }
        }
      }
      if (prm.fuse_reduce) {
        // Arrival: the CTA's partial stores are ordered before thread 0's
        // release (bar.sync, then a gpu-scope acq_rel fence before the atomic);
        // the last arriver's acquire fence orders the others' partials before
        // its reads, which bar.sync extends to the whole CTA.
        __shared__ int s_last;
        epi_bar_sync();
        const unsigned tile_id = blockIdx.z * gridDim.y + blockIdx.y;
        if (threadIdx.x == 0) {
          const unsigned prev = atomic_add_release_gpu(&prm.counters[tile_id], 1u);
          const bool last = prev == (unsigned)(prm.split_k - 1);
          if (last) fence_acq_rel_gpu();
          s_last = last;
        }
        epi_bar_sync();
        if (s_last && m_tile <= 2) {
          // One or two tokens: every thread loads its row's partials of all
          // splits at once straight from L2, summed in split order (as the
          // reduction kernel does).
          const int o = o0 + o_local;
          float b[4];
  #pragma unroll
          for (int a = 0; a < 4; ++a) b[a] = to_f32(bias_raw[a]);
          for (int tok = 0; tok < m_tile; ++tok) {
            float4 vs[kTcMaxSplit];
  #pragma unroll
            for (int sp = 0; sp < kTcMaxSplit; ++sp)
              vs[sp] = sp < prm.split_k ? ld_cg_f4(prm.partials + (size_t)sp * slot_stride + tile_off +
                                                 tok * kTcBlockO + o_local)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  #pragma unroll
            for (int sp = 0; sp < kTcMaxSplit; ++sp) {
              acc.x += vs[sp].x; acc.y += vs[sp].y; acc.z += vs[sp].z; acc.w += vs[sp].w;
            }
            if (ok && o < prm.N_g) {
              store_out<T, PEERS>(y, prm.peers, (int64_t)(t0 + tok) * prm.ld_y + 4 * o,
                           pack4<T>(acc.x + b[0], acc.y + b[1], acc.z + b[2], acc.w + b[3]));
            }
          }
          if (threadIdx.x == 0) prm.counters[tile_id] = 0u;
        } else if (s_last) {
          // Three or four tokens: every split's partials of this tile
          // ([token][row] float4, the real tokens only) are pulled into the
          // now idle stage buffers by bulk copies completing on one barrier,
          // one round trip for all of them, and summed in split order.
          const uint32_t slot_bytes = (uint32_t)(m_tile * kTcBlockO * 16);
          float4* red = reinterpret_cast<float4*>(smem);
          bool have = ok;
          if (threadIdx.x == 0 && ok) {
            asm volatile("fence.proxy.async.global;" ::: "memory");  // generic-proxy partials -> bulk copy
            mbar_arrive_expect_tx(red_full, slot_bytes * prm.split_k);
            for (int sp = 0; sp < prm.split_k; ++sp)
              bulk_load(smem + sp * slot_bytes, prm.partials + (size_t)sp * slot_stride + tile_off, slot_bytes,
                        red_full);
          }
          if (ok) have = mbar_wait(red_full, 0);
          const int o = o0 + o_local;
          float b[4];
  #pragma unroll
          for (int a = 0; a < 4; ++a) b[a] = to_f32(bias_raw[a]);
          for (int tok = 0; tok < m_tile; ++tok) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int sp = 0; sp < prm.split_k; ++sp) {
              const float4 v = red[(sp * m_tile + tok) * kTcBlockO + o_local];
              acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            }
            if (have && o < prm.N_g) {
              store_out<T, PEERS>(y, prm.peers, (int64_t)(t0 + tok) * prm.ld_y + 4 * o,
                           pack4<T>(acc.x + b[0], acc.y + b[1], acc.z + b[2], acc.w + b[3]));
            }
          }
          if (threadIdx.x == 0) prm.counters[tile_id] = 0u;
        }
      }
    }
  }

  // Outputs stored to peers are performed at system scope before the CTA
  // ends, so the barrier kernel that follows may signal them.
  if (PEERS) fence_sys();

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  // No CTA of a cluster leaves while a bulk copy may still read its send
  // buffer or write its receive buffer: an owner arrives once every partial
  // of its tokens has landed.  The arrive is relaxed: the barrier orders no
  // global stores (a release arrive waited for the output stores to complete).
  if (CLUSTER) {
    cluster_arrive_relaxed();
    cluster_wait_acquire();
  }
  if (threadIdx.x == 0 && *abort_flag) {
    // Let TMA loads that were issued but never consumed land before exiting.
    for (int it = *consumed_count; it < *issued_count; ++it)
      mbar_wait(&full[it % S], (it / S) & 1, 50000000ull);
    if (LORA == kLoraSimt) mbar_wait(t_full, 0, 50000000ull);  // the lora_a slice
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// Split-K reduction: y[m, 4o..4o+3] = round(sum over the split of the fp32
// partials + bias).  Launched as a programmatic dependent of the main kernel;
// it waits for the main grid to finish before reading the partials (the bias
// is read before that only when the caller declared the weights static).
template <typename T>
__global__ void __launch_bounds__(256)
qlin_splitk_reduce_kernel(const float4* __restrict__ partials, int split, int t_blocks, int o_blocks,
                          int n_tok, const T* __restrict__ bias, T* __restrict__ y, int64_t ld_y, int M,
                          int N_g, int static_weights, const PeerOut peers) {
  pdl_launch_dependents();
  const int64_t per_slot = (int64_t)t_blocks * o_blocks * n_tok * kTcBlockO;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = idx < per_slot;
  // idx -> (t-block, o-block, token, row) in the partials' layout
  const int row = (int)(idx % kTcBlockO);
  const int tok = (int)((idx / kTcBlockO) % n_tok);
  const int ob = (int)((idx / ((int64_t)kTcBlockO * n_tok)) % o_blocks);
  const int tb = (int)(idx / ((int64_t)kTcBlockO * n_tok * o_blocks));
  const int o = ob * kTcBlockO + row, m = tb * n_tok + tok;
  const bool valid = live && o < N_g && m < M;
  T braw[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) braw[a] = from_f32<T>(0.f);
  if (static_weights && valid && bias) {
#pragma unroll
    for (int a = 0; a < 4; ++a) braw[a] = bias[4 * o + a];
  }
  pdl_wait_prior();
  if (!valid) return;
  if (!static_weights && bias) {
#pragma unroll
    for (int a = 0; a < 4; ++a) braw[a] = bias[4 * o + a];
  }
  // All slots are loaded before any is summed, so the loads are in flight
  // together rather than one L2 round trip per slot.
  float4 v[kTcMaxSplit];
#pragma unroll
  for (int s = 0; s < kTcMaxSplit; ++s)
    v[s] = s < split ? partials[s * per_slot + idx] : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int s = 0; s < kTcMaxSplit; ++s) {
    acc.x += v[s].x; acc.y += v[s].y; acc.z += v[s].z; acc.w += v[s].w;
  }
  float b[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) b[a] = to_f32(braw[a]);
  store_out<T, true>(y, peers, (int64_t)m * ld_y + 4 * o,
                     pack4<T>(acc.x + b[0], acc.y + b[1], acc.z + b[2], acc.w + b[3]));
  if (has_peers(peers)) fence_sys();
}

}  // namespace qlin
