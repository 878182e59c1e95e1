// CUDA-core kernels of the quaternion linear path:
//  * qlin_simt_kernel      -- tiled Hamilton-product GEMM on FMA units (fp32, and
//                             the fallback for bf16/f16 shapes the tensor-core
//                             path does not take); fp32 accumulation.
//  * qlin_lora_down_kernel -- t = x A^T for the fused LoRA residual.
//  * qlin_planarize_kernel -- x[m, 4i+q] -> xp[q][m][i] (component planes), the
//                             operand layout of the tensor-core kernel.
//  * qlin_prologue_kernel  -- the tensor-core path's prologue: component planes
//                             and the scaled LoRA down projection in one launch.
//  * qlin_gather_kernel    -- [G, M, n] shards -> [M, G*n] columns.
#pragma once

#include "qlin_common.cuh"

namespace qlin {

// y[m, 4o+a] = sum_i (W[o,i] (x) X[m,i])_a (+ bias) (+ scale * t[m,:] . B[4o+a,:])
// Tile: BM tokens x BO output quaternions, BK input quaternions per step.
// Thread (tx, ty) owns tokens ty + 16*t (t < TM) and outputs tx + 16*j (j < TO).
template <typename T, int BM, int BO, int BK, int TM, int TO>
__global__ void __launch_bounds__((BM / TM) * (BO / TO))
qlin_simt_kernel(const T* __restrict__ x, int64_t ld_x,
                 const T* __restrict__ wr, const T* __restrict__ wi,
                 const T* __restrict__ wj, const T* __restrict__ wk, int64_t ld_w,
                 const T* __restrict__ bias,
                 const float* __restrict__ lora_t, const T* __restrict__ lora_b, int rank,
                 float lora_scale,
                 T* __restrict__ y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g) {
  constexpr int TX = BO / TO, TY = BM / TM, NT = TX * TY;
  static_assert(TX == 16 && TY == 16, "thread grid is 16 x 16");
  __shared__ float4 xs[BK][BM];
  __shared__ float4 ws[BK][BO];

  const int tid = threadIdx.y * TX + threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * BM;
  const int64_t o0 = (int64_t)blockIdx.x * BO;
  const T* wp[4] = {wr, wi, wj, wk};

  float acc[TM][TO][4];
#pragma unroll
  for (int t = 0; t < TM; ++t)
#pragma unroll
    for (int j = 0; j < TO; ++j)
#pragma unroll
      for (int a = 0; a < 4; ++a) acc[t][j][a] = 0.f;

  float* xsf = reinterpret_cast<float*>(&xs[0][0]);
  float* wsf = reinterpret_cast<float*>(&ws[0][0]);

  for (int64_t i0 = 0; i0 < K_g; i0 += BK) {
    // x tile: BM rows of 4*BK consecutive elements.
    for (int idx = tid; idx < BM * BK * 4; idx += NT) {
      const int mm = idx / (BK * 4), rem = idx % (BK * 4);
      const int ii = rem >> 2, q = rem & 3;
      const int64_t m = m0 + mm, i = i0 + ii;
      float v = 0.f;
      if (m < M && i < K_g) v = to_f32(x[m * ld_x + 4 * i + q]);
      xsf[(ii * BM + mm) * 4 + q] = v;
    }
    // weight tiles: component p, BO rows of BK consecutive input groups.
    for (int idx = tid; idx < 4 * BO * BK; idx += NT) {
      const int p = idx / (BO * BK), rem = idx % (BO * BK);
      const int oo = rem / BK, ii = rem % BK;
      const int64_t o = o0 + oo, i = i0 + ii;
      float v = 0.f;
      if (o < N_g && i < K_g) v = to_f32(wp[p][o * ld_w + i]);
      wsf[(ii * BO + oo) * 4 + p] = v;
    }
    __syncthreads();
#pragma unroll 4
    for (int ii = 0; ii < BK; ++ii) {
      float4 xv[TM], wv[TO];
#pragma unroll
      for (int t = 0; t < TM; ++t) xv[t] = xs[ii][threadIdx.y + 16 * t];
#pragma unroll
      for (int j = 0; j < TO; ++j) wv[j] = ws[ii][threadIdx.x + 16 * j];
#pragma unroll
      for (int t = 0; t < TM; ++t)
#pragma unroll
        for (int j = 0; j < TO; ++j) {
          const float4 w = wv[j], q = xv[t];
          // Hamilton product w (x) q (reference quaternion/reference.py:41-44)
          acc[t][j][0] += w.x * q.x - w.y * q.y - w.z * q.z - w.w * q.w;
          acc[t][j][1] += w.x * q.y + w.y * q.x + w.z * q.w - w.w * q.z;
          acc[t][j][2] += w.x * q.z - w.y * q.w + w.z * q.x + w.w * q.y;
          acc[t][j][3] += w.x * q.w + w.y * q.z - w.z * q.y + w.w * q.x;
        }
    }
    __syncthreads();
  }

#pragma unroll
  for (int t = 0; t < TM; ++t) {
    const int64_t m = m0 + threadIdx.y + 16 * t;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TO; ++j) {
      const int64_t o = o0 + threadIdx.x + 16 * j;
      if (o >= N_g) continue;
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int64_t n = 4 * o + a;
        float v = acc[t][j][a];
        if (bias) v += to_f32(bias[n]);
        if (rank > 0) {
          float l = 0.f;
          for (int r = 0; r < rank; ++r) l += lora_t[m * rank + r] * to_f32(lora_b[n * rank + r]);
          v += lora_scale * l;
        }
        y[m * ld_y + n] = from_f32<T>(v);
      }
    }
  }
}

// t[m, r] = sum_k x[m,k] * A[r,k].  One warp per rank row r, TOKS tokens per
// block; fp32 accumulate.  Writes t_f32 (unscaled, [M, rank]) and/or t_tc
// (scaled by lora_scale, rounded to T, [M, ld_t]) when those are non-null.
template <typename T, int TOKS>
__global__ void __launch_bounds__(256)
qlin_lora_down_kernel(const T* __restrict__ x, int64_t ld_x, const T* __restrict__ lora_a, int rank,
                      int64_t M, int64_t K, float lora_scale, float* __restrict__ t_f32,
                      T* __restrict__ t_tc, int64_t ld_t) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.y * 8 + warp;
  const int64_t m0 = (int64_t)blockIdx.x * TOKS;
  if (r >= rank) return;
  float acc[TOKS];
#pragma unroll
  for (int t = 0; t < TOKS; ++t) acc[t] = 0.f;
  const T* arow = lora_a + (int64_t)r * K;
  for (int64_t k = lane; k < K; k += 32) {
    const float a = to_f32(arow[k]);
#pragma unroll
    for (int t = 0; t < TOKS; ++t)
      if (m0 + t < M) acc[t] += a * to_f32(x[(m0 + t) * ld_x + k]);
  }
#pragma unroll
  for (int t = 0; t < TOKS; ++t) {
    float v = acc[t];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    acc[t] = v;
  }
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < TOKS; ++t) {
      const int64_t m = m0 + t;
      if (m >= M) break;
      if (t_f32) t_f32[m * rank + r] = acc[t];
      if (t_tc) t_tc[m * ld_t + r] = from_f32<T>(lora_scale * acc[t]);
    }
  }
}

// Component planes of x: xp[q * M * K_g + m * K_g + i] = x[m * ld_x + 4i + q].
// One thread moves 8 quaternions (64 bytes in, 4 x 16 bytes out).
// Requires K_g % 8 == 0, ld_x % 8 == 0 and 16-byte aligned x and xp.
template <typename T>
__global__ void __launch_bounds__(256)
qlin_planarize_kernel(const T* __restrict__ x, int64_t ld_x, T* __restrict__ xp, int64_t M,
                      int64_t K_g) {
  static_assert(sizeof(T) == 2, "planarize moves 16-bit elements");
  const int64_t groups = K_g / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= M * groups) return;
  const int64_t m = idx / groups, g = idx % groups;
  const uint4* src = reinterpret_cast<const uint4*>(x + m * ld_x + 32 * g);
  uint32_t w[16];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 v = ld_cg_v4(src + c);
    w[4 * c + 0] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
  }
  // word 2j holds components (r, i) of quaternion j, word 2j+1 holds (j, k).
  uint32_t out[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t a0 = w[4 * j], a1 = w[4 * j + 1], b0 = w[4 * j + 2], b1 = w[4 * j + 3];
    out[0][j] = __byte_perm(a0, b0, 0x5410);
    out[1][j] = __byte_perm(a0, b0, 0x7632);
    out[2][j] = __byte_perm(a1, b1, 0x5410);
    out[3][j] = __byte_perm(a1, b1, 0x7632);
  }
  const int64_t plane = M * K_g;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4* dst = reinterpret_cast<uint4*>(xp + q * plane + m * K_g + 8 * g);
    *dst = make_uint4(out[q][0], out[q][1], out[q][2], out[q][3]);
  }
}

// Prologue of the tensor-core path, one launch:
//  * blocks [0, planar_blocks): component planes of x (as qlin_planarize_kernel);
//  * the remaining blocks: scaled LoRA down projection
//      t[m, r] = lora_scale * sum_k x[m, k] A[r, k]
//    one block per (8 tokens, RR ranks), threads striding over K in 8-element
//    (16-byte) vectors, fp32 accumulation, rounded to T once.  RR = 1 spreads
//    a few tokens over many blocks; RR = 8 reuses each x row for 8 ranks.
// Launched as a programmatic dependent of the previous kernel of the stream:
// it waits for that kernel, then lets the next kernel (this call's main
// kernel) launch, so that the main kernel's launch implies that all earlier
// work of the stream is complete.  Requires K % 8 == 0 and 16-byte aligned x,
// lora_a and rows (ld_x % 8 == 0).
template <typename T, int RR>
__global__ void __launch_bounds__(256)
qlin_prologue_kernel(const T* __restrict__ x, int64_t ld_x, T* __restrict__ xp, int64_t M, int64_t K_g,
                     int64_t planar_blocks, const T* __restrict__ lora_a, int rank, float lora_scale,
                     T* __restrict__ t_tc, int64_t ld_t) {
  static_assert(sizeof(T) == 2, "16-bit elements");
  pdl_wait_prior();
  pdl_launch_dependents();
  if ((int64_t)blockIdx.x < planar_blocks) {
    const int64_t groups = K_g / 8;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= M * groups) return;
    const int64_t m = idx / groups, g = idx % groups;
    const uint4* src = reinterpret_cast<const uint4*>(x + m * ld_x + 32 * g);
    uint32_t w[16];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 v = ld_cg_v4(src + c);
      w[4 * c + 0] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
    }
    const int64_t plane = M * K_g;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t a = w[4 * j + (q >> 1)], b = w[4 * j + 2 + (q >> 1)];
        o[j] = __byte_perm(a, b, (q & 1) ? 0x7632 : 0x5410);
      }
      *reinterpret_cast<uint4*>(xp + q * plane + m * K_g + 8 * g) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    return;
  }
  constexpr int TT = 8;
  const int64_t b = (int64_t)blockIdx.x - planar_blocks;
  const int rblocks = (rank + RR - 1) / RR;
  const int64_t m0 = (b / rblocks) * TT;
  const int r0 = (int)(b % rblocks) * RR;
  const int64_t K = 4 * K_g, nvec = K / 8;
  float acc[TT][RR];
#pragma unroll
  for (int t = 0; t < TT; ++t)
#pragma unroll
    for (int r = 0; r < RR; ++r) acc[t][r] = 0.f;
  // U 8-element vectors per thread and step (2 for RR = 1), all of a step's
  // loads issued before any is used: a 4096-wide decode row is then one step
  // of 256 threads, one memory round trip.
  constexpr int U = RR == 1 ? 2 : 1;
  for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += U * (int64_t)blockDim.x) {
    uint4 ua[U][RR];
#pragma unroll
    for (int h = 0; h < U; ++h) {
      const int64_t v = v0 + h * (int64_t)blockDim.x;
#pragma unroll
      for (int r = 0; r < RR; ++r)
        ua[h][r] = (v < nvec && r0 + r < rank)
                       ? ld_cg_v4(reinterpret_cast<const uint4*>(lora_a + (int64_t)(r0 + r) * K) + v)
                       : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      if (m0 + t >= M) break;
      uint4 ux[U];
#pragma unroll
      for (int h = 0; h < U; ++h) {
        const int64_t v = v0 + h * (int64_t)blockDim.x;
        ux[h] = v < nvec ? ld_cg_v4(reinterpret_cast<const uint4*>(x + (m0 + t) * ld_x) + v)
                         : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int h = 0; h < U; ++h) {
        const T* e = reinterpret_cast<const T*>(&ux[h]);
        float xv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[j] = to_f32(e[j]);
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          const T* ea = reinterpret_cast<const T*>(&ua[h][r]);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[t][r] += to_f32(ea[j]) * xv[j];
        }
      }
    }
  }
  __shared__ float red[8][TT * RR];
  static_assert(TT * RR <= 256, "one thread per reduced value");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int t = 0; t < TT; ++t)
#pragma unroll
    for (int r = 0; r < RR; ++r) {
      float s = acc[t][r];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0) red[warp][t * RR + r] = s;
    }
  __syncthreads();
  if (threadIdx.x < TT * RR) {
    const int t = threadIdx.x / RR, r = threadIdx.x % RR;
    float s = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < 8; ++w2) s += red[w2][threadIdx.x];
    if (m0 + t < M && r0 + r < rank) t_tc[(m0 + t) * ld_t + r0 + r] = from_f32<T>(lora_scale * s);
  }
}

// dst[m * ld_dst + g * n + j] = src[(g * M + m) * n + j]
template <typename E>
__global__ void __launch_bounds__(256)
qlin_gather_kernel(const E* __restrict__ src, E* __restrict__ dst, int64_t G, int64_t M, int64_t n,
                   int64_t ld_dst) {
  const int64_t total = G * M * n;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = idx % n, gm = idx / n;
    const int64_t m = gm % M, g = gm / M;
    dst[m * ld_dst + g * n + j] = src[idx];
  }
}

// Cross-rank barrier of the column-partitioned layer.  It runs twice per
// call: before the shard kernel (entry: every rank has finished the work it
// queued after the previous call, so nobody still reads an output that this
// call overwrites) and after it (exit: every rank's columns have landed in
// every rank's output).  One warp: lane p (p != rank) writes this barrier's
// epoch into slot `slot0 + rank` of rank p's flag array (release, system
// scope), then waits -- bounded -- until slot `slot0 + p` of this rank's
// array holds the epoch (acquire, system scope).  Each barrier has its own
// slots and its own per-rank device counter, advanced here, so every rank,
// taking the same sequence of calls, agrees on the epochs without host
// involvement (CUDA graphs replay them unchanged).  A wait that runs out
// records QLIN_ERR_TIMEOUT and returns.
struct PeerFlags {
  unsigned* f[kMaxPeers + 1];  // flag array [2 * world] of every rank, by rank
};

__global__ void __launch_bounds__(32) qlin_peer_barrier_kernel(const PeerFlags pf, unsigned* epoch_word,
                                                               int rank, int world, int slot0) {
  __shared__ unsigned e;
  if (threadIdx.x == 0) {
    e = *epoch_word + 1u;
    *epoch_word = e;
  }
  __syncwarp();
  const unsigned ep = e;
  const int p = threadIdx.x;
  if (p < world && p != rank) {
    fence_sys();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(pf.f[p] + slot0 + rank), "r"(ep) : "memory");
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(pf.f[rank] + slot0 + p) : "memory");
      if ((int)(v - ep) >= 0) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_error(7);
        break;
      }
    }
  }
}

}  // namespace qlin
