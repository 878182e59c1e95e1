// Tensor-core quaternion linear forward for sm_100a (TMA + tcgen05 + TMEM).
//
// Decomposition.  With component planes X_q[m, i] = x[m, 4i+q] (written by
// qlin_planarize_kernel) the Hamilton-product layer is sixteen real products
//
//     Y_a[m, o] = sum_p s(a,p) * sum_i W_p[o, i] * X_{p^a}[m, i]
//
// (a = output component, p = weight component, q = p XOR a is the input
// component it pairs with, s(a,p) = +-1 is the sign of the 4x4 block matrix
// of reference quaternion/packing.py:18-21).  Each (a, p) term is one UMMA
// whose A operand is a W_p tile exactly as TMA loads it from the caller's
// weight tensor and whose B operand is an X_q tile; the sign is the
// instruction descriptor's negate-A bit.  The four output components
// accumulate in four fp32 TMEM accumulators.  Nothing is expanded: every
// weight byte crosses HBM once per tile, a quarter of a dense layer's.
//
// CTA tile: 128 output quaternions (UMMA M = 128, one TMEM lane each) x
// N_TOK tokens (UMMA N) x all four components.  K is walked in chunks of 32
// input quaternions (64-byte rows, 64-byte TMA/UMMA swizzle).  For few tiles
// (decode) the K chunks of one tile are split over the CTAs of a cluster and
// the fp32 partials are summed through distributed shared memory.
//
// Roles (128 threads): thread 0 issues TMA, warp 1 owns TMEM and its lane 0
// issues UMMA, all four warps run the epilogue (warp w reads TMEM lanes
// 32w..32w+31).  Every mbarrier wait is bounded (qlin_common.cuh).
#pragma once

#include "qlin_common.cuh"

namespace qlin {

constexpr int kTcBlockO = 128;   // output quaternions per CTA tile (UMMA M)
constexpr int kTcChunk = 32;     // input quaternions per K chunk (64-byte rows)
constexpr int kTcThreads = 128;
constexpr int kTcWTileBytes = kTcBlockO * kTcChunk * 2;  // 8 KB

template <int N_TOK>
struct TcCfg {
  static constexpr int kXTileBytes = N_TOK * kTcChunk * 2;
  static constexpr int kStageBytes = 4 * kTcWTileBytes + 4 * kXTileBytes;
  static constexpr int kStages = N_TOK >= 128 ? 3 : (N_TOK >= 64 ? 4 : (N_TOK >= 32 ? 5 : 6));
  static constexpr int kTmemCols = 4 * N_TOK;  // 64 .. 512, power of two
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // + barriers + alignment slack
  static_assert(N_TOK == 16 || N_TOK == 32 || N_TOK == 64 || N_TOK == 128, "UMMA N");
  // Split-K partials (4 * N_TOK * 128 fp32) reuse the stage buffers.
  static constexpr bool kAllowSplit = 4 * N_TOK * 128 * 4 <= kStages * kStageBytes;
};

// neg(a, p): sign of W_p in output component a (rows of packing.py:18-21).
__host__ __device__ constexpr bool quat_neg(int a, int p) {
  return (a == 0 && p != 0) || (a == 1 && p == 3) || (a == 2 && p == 1) || (a == 3 && p == 2);
}

struct TcParams {
  const void* bias;   // [4*N_g] or null
  void* y;            // [M, ld_y]
  int64_t ld_y;
  int M, N_g;
  int num_chunks;     // ceil(K_g / 32)
  int lora_chunks;    // ceil(rank / 32), 0 without LoRA
  int split_k;        // CTAs per cluster along K (1 = no split)
};

template <typename T, int N_TOK>
__global__ void __launch_bounds__(kTcThreads, 1)
qlin_tc_kernel(const __grid_constant__ CUtensorMap map_wr, const __grid_constant__ CUtensorMap map_wi,
               const __grid_constant__ CUtensorMap map_wj, const __grid_constant__ CUtensorMap map_wk,
               const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_lb,
               const __grid_constant__ CUtensorMap map_t, const TcParams prm) {
  using Cfg = TcCfg<N_TOK>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescPos = make_idesc_f16(128, N_TOK, kFmt, false);
  constexpr uint32_t kIdescNeg = make_idesc_f16(128, N_TOK, kFmt, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_count = const_cast<int*>(abort_flag) + 1;
  int* consumed_count = issued_count + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = blockIdx.y * kTcBlockO;
  const int t0 = blockIdx.z * N_TOK;
  const int ks = blockIdx.x;  // K split index == rank in the cluster
  const int c_begin = (int)((int64_t)ks * prm.num_chunks / prm.split_k);
  const int c_end = (int)((int64_t)(ks + 1) * prm.num_chunks / prm.split_k);
  const int my_main = c_end - c_begin;
  const int my_lora = (ks == prm.split_k - 1) ? prm.lora_chunks : 0;
  const int total = my_main + my_lora;

  auto w_tile = [&](int s, int p) { return smem + s * Cfg::kStageBytes + p * kTcWTileBytes; };
  auto x_tile = [&](int s, int q) {
    return smem + s * Cfg::kStageBytes + 4 * kTcWTileBytes + q * Cfg::kXTileBytes;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *issued_count = 0;
    *consumed_count = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_wr);
    tma_prefetch_desc(&map_wi);
    tma_prefetch_desc(&map_wj);
    tma_prefetch_desc(&map_wk);
    tma_prefetch_desc(&map_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (threadIdx.x == 0) {
    // ---------------- TMA producer ----------------
    const CUtensorMap* wmap[4] = {&map_wr, &map_wi, &map_wj, &map_wk};
    int it = 0;
    for (; it < total; ++it) {
      const int s = it % S, n = it / S;
      if (it >= S && !mbar_wait(&empty[s], (n - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      if (it < my_main) {
        const int k = (c_begin + it) * kTcChunk;
        mbar_arrive_expect_tx(&full[s], 4 * kTcWTileBytes + 4 * Cfg::kXTileBytes);
#pragma unroll
        for (int p = 0; p < 4; ++p) tma_load_2d(w_tile(s, p), wmap[p], &full[s], k, o0);
#pragma unroll
        for (int q = 0; q < 4; ++q) tma_load_3d(x_tile(s, q), &map_x, &full[s], k, t0, q);
      } else {
        const int r = (it - my_main) * kTcChunk;
        mbar_arrive_expect_tx(&full[s], 4 * kTcWTileBytes + Cfg::kXTileBytes);
#pragma unroll
        for (int a = 0; a < 4; ++a) tma_load_3d(w_tile(s, a), &map_lb, &full[s], r, a, o0);
        tma_load_2d(x_tile(s, 0), &map_t, &full[s], r, t0);
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
#pragma unroll
            for (int a = 0; a < 4; ++a) {
              const uint64_t bdesc = smem_desc_sw64(x_tile(s, p ^ a)) + 2 * kk;
              umma_f16(tmem_base + a * N_TOK, adesc, bdesc, quat_neg(a, p) ? kIdescNeg : kIdescPos,
                       (it > 0 || kk > 0 || p > 0) ? 1u : 0u);
            }
          }
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
    }
    *consumed_count = it;
    umma_commit(acc_full);  // fires once every UMMA issued above has completed
  }
  __syncwarp();

  // ---------------- epilogue ----------------
  const bool acc_ok = mbar_wait(acc_full, 0);
  tc_fence_after();
  const bool ok = acc_ok && (*abort_flag == 0);
  const int o_local = warp * 32 + lane;
  const uint32_t lane_addr = tmem_base + ((uint32_t)(warp * 32) << 16);
  T* __restrict__ y = reinterpret_cast<T*>(prm.y);
  const T* __restrict__ bias = reinterpret_cast<const T*>(prm.bias);

  if (prm.split_k == 1) {
    const int o = o0 + o_local;
    float b[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok && bias && o < prm.N_g) {
#pragma unroll
      for (int a = 0; a < 4; ++a) b[a] = to_f32(bias[4 * o + a]);
    }
#pragma unroll 1
    for (int j = 0; j < N_TOK / 16; ++j) {
      float v[4][16];
#pragma unroll
      for (int a = 0; a < 4; ++a) tmem_ld16(lane_addr + a * N_TOK + j * 16, v[a]);
      tmem_ld_wait();
      if (ok && o < prm.N_g) {
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const int m = t0 + j * 16 + t;
          if (m < prm.M) {
            *reinterpret_cast<uint2*>(y + (int64_t)m * prm.ld_y + 4 * o) =
                pack4<T>(v[0][t] + b[0], v[1][t] + b[1], v[2][t] + b[2], v[3][t] + b[3]);
          }
        }
      }
    }
  } else {
    // Partials -> own shared memory as red[(a*N_TOK + tok) * 128 + o_local].
    float* red = reinterpret_cast<float*>(smem);
    const bool smem_free = ok;  // all loads were consumed by completed UMMAs
#pragma unroll 1
    for (int j = 0; j < N_TOK / 16; ++j) {
      float v[4][16];
#pragma unroll
      for (int a = 0; a < 4; ++a) tmem_ld16(lane_addr + a * N_TOK + j * 16, v[a]);
      tmem_ld_wait();
      if (smem_free) {
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int t = 0; t < 16; ++t) red[(a * N_TOK + j * 16 + t) * 128 + o_local] = v[a][t];
      }
    }
    cluster_sync_all();
    // CTA `ks` finalises output rows [ks*rows, (ks+1)*rows) of the tile.
    const int rows = kTcBlockO / prm.split_k;
    const uint32_t red_addr = smem_u32(red);
    int all_ok = ok ? 1 : 0;
    for (int idx = threadIdx.x; idx < rows * N_TOK; idx += kTcThreads) {
      const int ol = ks * rows + idx % rows, tok = idx / rows;
      const int o = o0 + ol, m = t0 + tok;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int peer = 0; peer < prm.split_k; ++peer) {
        const uint32_t base = map_peer_smem(red_addr, (uint32_t)peer);
#pragma unroll
        for (int a = 0; a < 4; ++a) acc[a] += ld_peer_f32(base + (uint32_t)(((a * N_TOK + tok) * 128 + ol) * 4));
      }
      if (all_ok && o < prm.N_g && m < prm.M) {
        float b[4] = {0.f, 0.f, 0.f, 0.f};
        if (bias) {
#pragma unroll
          for (int a = 0; a < 4; ++a) b[a] = to_f32(bias[4 * o + a]);
        }
        *reinterpret_cast<uint2*>(y + (int64_t)m * prm.ld_y + 4 * o) =
            pack4<T>(acc[0] + b[0], acc[1] + b[1], acc[2] + b[2], acc[3] + b[3]);
      }
    }
    cluster_sync_all();  // peers may still read this CTA's partials until here
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // Let TMA loads that were issued but never consumed land before exiting.
    for (int it = *consumed_count; it < *issued_count; ++it)
      mbar_wait(&full[it % S], (it / S) & 1, 50000000ull);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace qlin
