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
//  * qlin_stage_in_kernel  -- qlin_forward_host's small copy of x from
//                             page-locked host memory to the device.
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

// fp32 Hamilton-product GEMM on CUDA cores with a K split (fp32 layers: the
// 1e-5 relative error bound of an fp32 layer needs FFMA, not TF32).
//
// CTA tile: 64 tokens x 32 output quaternions; thread (tx, ty) of 16 x 16
// owns tokens ty + 16 t (t < 4) and output quaternions tx + 16 j (j < 2): 128
// FMAs per input quaternion from 6 shared-memory float4 reads.  Input
// quaternions [k0, k1) of this split are walked 8 at a time through two
// shared-memory buffers: the next step's x quaternions (one float4 each) and
// W pieces (4 consecutive inputs of one component row, one float4) are loaded
// into registers while the current step computes.  The fp32 partial of the
// split goes to part[split][M][4 N_g] (or, with one split, straight to y with
// bias and the LoRA up projection); qlin_splitk_f32_reduce_kernel sums the
// splits in order.  Requires 16-byte aligned x and weights, ld_x and ld_w
// multiples of 4 (float4 loads).
constexpr int kSkBM = 64, kSkBO = 32, kSkBK = 8, kSkTM = 4, kSkTO = 2;

__device__ __forceinline__ void hamilton_acc(float (&acc)[4], const float4 w, const float4 q) {
  // w (x) q (reference quaternion/reference.py:41-44)
  acc[0] = fmaf(w.x, q.x, acc[0]); acc[0] = fmaf(-w.y, q.y, acc[0]); acc[0] = fmaf(-w.z, q.z, acc[0]); acc[0] = fmaf(-w.w, q.w, acc[0]);
  acc[1] = fmaf(w.x, q.y, acc[1]); acc[1] = fmaf(w.y, q.x, acc[1]); acc[1] = fmaf(w.z, q.w, acc[1]); acc[1] = fmaf(-w.w, q.z, acc[1]);
  acc[2] = fmaf(w.x, q.z, acc[2]); acc[2] = fmaf(-w.y, q.w, acc[2]); acc[2] = fmaf(w.z, q.x, acc[2]); acc[2] = fmaf(w.w, q.y, acc[2]);
  acc[3] = fmaf(w.x, q.w, acc[3]); acc[3] = fmaf(w.y, q.z, acc[3]); acc[3] = fmaf(-w.z, q.y, acc[3]); acc[3] = fmaf(w.w, q.x, acc[3]);
}

__global__ void __launch_bounds__(256)
qlin_simt_splitk_kernel(const float* __restrict__ x, int64_t ld_x, const float* __restrict__ wr,
                        const float* __restrict__ wi, const float* __restrict__ wj, const float* __restrict__ wk,
                        int64_t ld_w, const float* __restrict__ bias, const float* __restrict__ lora_t,
                        const float* __restrict__ lora_b, int rank, float lora_scale, float* __restrict__ y,
                        int64_t ld_y, float* __restrict__ part, int M, int K_g, int N_g, int split) {
  __shared__ float4 xs[2][kSkBK][kSkBM];
  __shared__ float4 ws[2][kSkBK][kSkBO];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4, tid = threadIdx.x;
  const int m0 = blockIdx.y * kSkBM, o0 = blockIdx.x * kSkBO, sp = blockIdx.z;
  // whole 8-quaternion steps per split, so every float4 load is 16-byte aligned
  const int nst = (K_g + kSkBK - 1) / kSkBK;
  const int k0 = kSkBK * (int)((int64_t)sp * nst / split);
  const int k1 = min(K_g, kSkBK * (int)((int64_t)(sp + 1) * nst / split));
  // this thread's loads of one step: x quaternions (m = tid/8 + 32 h, k = tid%8)
  // and one W piece (component p, row o, inputs kg*4 .. kg*4+3)
  const int xm = tid >> 3, xk = tid & 7;
  const int wpc = tid >> 6, wo = (tid >> 1) & 31, wkg = tid & 1;
  const float* wsrc_row = wpc == 0 ? wr : (wpc == 1 ? wi : (wpc == 2 ? wj : wk));
  float4 rx[2], rw;
  auto load_step = [&](int kb) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = m0 + xm + 32 * h, k = kb + xk;
      rx[h] = (m < M && k < k1) ? ld_cg_f4(x + (int64_t)m * ld_x + 4 * (int64_t)k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int o = o0 + wo, k = kb + 4 * wkg;
    const float* src = wsrc_row + (int64_t)o * ld_w + k;
    if (o < N_g && k + 3 < k1) {
      rw = ld_cg_f4(src);
    } else {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = (o < N_g && k + i < k1) ? src[i] : 0.f;
      rw = make_float4(v[0], v[1], v[2], v[3]);
    }
  };
  auto store_step = [&](int buf) {
#pragma unroll
    for (int h = 0; h < 2; ++h) xs[buf][xk][xm + 32 * h] = rx[h];
    float* wsf = reinterpret_cast<float*>(&ws[buf][0][0]) + (4 * wkg * kSkBO + wo) * 4 + wpc;
    wsf[0 * kSkBO * 4] = rw.x;
    wsf[1 * kSkBO * 4] = rw.y;
    wsf[2 * kSkBO * 4] = rw.z;
    wsf[3 * kSkBO * 4] = rw.w;
  };

  float acc[kSkTM][kSkTO][4];
#pragma unroll
  for (int t = 0; t < kSkTM; ++t)
#pragma unroll
    for (int j = 0; j < kSkTO; ++j)
#pragma unroll
      for (int a = 0; a < 4; ++a) acc[t][j][a] = 0.f;

  int buf = 0;
  if (k0 < k1) {
    load_step(k0);
    store_step(0);
  }
  __syncthreads();
  for (int kb = k0; kb < k1; kb += kSkBK) {
    const bool more = kb + kSkBK < k1;
    if (more) load_step(kb + kSkBK);  // in flight during this step's math
#pragma unroll
    for (int k = 0; k < kSkBK; ++k) {
      float4 xv[kSkTM], wv[kSkTO];
#pragma unroll
      for (int t = 0; t < kSkTM; ++t) xv[t] = xs[buf][k][ty + 16 * t];
#pragma unroll
      for (int j = 0; j < kSkTO; ++j) wv[j] = ws[buf][k][tx + 16 * j];
#pragma unroll
      for (int t = 0; t < kSkTM; ++t)
#pragma unroll
        for (int j = 0; j < kSkTO; ++j) hamilton_acc(acc[t][j], wv[j], xv[t]);
    }
    if (more) store_step(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }

#pragma unroll
  for (int t = 0; t < kSkTM; ++t) {
    const int m = m0 + ty + 16 * t;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < kSkTO; ++j) {
      const int o = o0 + tx + 16 * j;
      if (o >= N_g) continue;
      float v[4] = {acc[t][j][0], acc[t][j][1], acc[t][j][2], acc[t][j][3]};
      if (split > 1) {
        *reinterpret_cast<float4*>(part + ((int64_t)sp * M + m) * (4 * (int64_t)N_g) + 4 * o) =
            make_float4(v[0], v[1], v[2], v[3]);
        continue;
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int64_t n = 4 * (int64_t)o + a;
        if (bias) v[a] += bias[n];
        if (rank > 0) {
          float l = 0.f;
          for (int r = 0; r < rank; ++r) l += lora_t[(int64_t)m * rank + r] * lora_b[n * rank + r];
          v[a] += lora_scale * l;
        }
      }
      *reinterpret_cast<float4*>(y + (int64_t)m * ld_y + 4 * o) = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
}

// y[m, 4o .. 4o+3] = sum over the splits, in order, of the fp32 partials
// + bias + lora_scale * t[m,:] . B[4o+a,:].  One thread per output quaternion.
__global__ void __launch_bounds__(256)
qlin_splitk_f32_reduce_kernel(const float* __restrict__ part, int split, const float* __restrict__ bias,
                              const float* __restrict__ lora_t, const float* __restrict__ lora_b, int rank,
                              float lora_scale, float* __restrict__ y, int64_t ld_y, int M, int N_g) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)M * N_g) return;
  const int m = (int)(idx / N_g), o = (int)(idx % N_g);
  const int64_t row = 4 * (int64_t)N_g;
  float4 acc = ld_cg_f4(part + (int64_t)m * row + 4 * o);
  for (int s = 1; s < split; ++s) {
    const float4 v = ld_cg_f4(part + ((int64_t)s * M + m) * row + 4 * o);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  const int64_t n0 = 4 * (int64_t)o;
  if (bias) {
    acc.x += bias[n0]; acc.y += bias[n0 + 1]; acc.z += bias[n0 + 2]; acc.w += bias[n0 + 3];
  }
  if (rank > 0) {
    float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
    const float* tr = lora_t + (int64_t)m * rank;
    for (int r = 0; r < rank; ++r) {
      const float t = tr[r];
      l0 = fmaf(t, lora_b[n0 * rank + r], l0);
      l1 = fmaf(t, lora_b[(n0 + 1) * rank + r], l1);
      l2 = fmaf(t, lora_b[(n0 + 2) * rank + r], l2);
      l3 = fmaf(t, lora_b[(n0 + 3) * rank + r], l3);
    }
    acc.x += lora_scale * l0; acc.y += lora_scale * l1; acc.z += lora_scale * l2; acc.w += lora_scale * l3;
  }
  *reinterpret_cast<float4*>(y + (int64_t)m * ld_y + n0) = acc;
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

// qlin_forward_host for decode-sized inputs: x comes from page-locked host
// memory (through its device mapping) by this kernel of the call's
// programmatic-dependent chain rather than by a copy-engine transfer
// (measured: an 8 KB cudaMemcpyAsync each way cost about 6 us of device time
// per call; a kernel's PCIe round trip about 1 us).  Rows of `row` 16-byte
// words, leading dimensions in 16-byte words, two words per thread.  The
// host reads are issued before the dependency wait (earlier work of the
// stream does not write the caller's host buffer; the host wrote it before
// the call), the device stores after it (earlier calls' kernels may still
// read the staging buffer).  Reads bypass the caches (ld.global.cv): the host
// rewrites the buffer between calls.
__global__ void __launch_bounds__(256)
qlin_stage_in_kernel(const uint4* __restrict__ src, int64_t ld_src, uint4* __restrict__ dst, int64_t ld_dst,
                     int64_t row, int64_t M) {
  pdl_launch_dependents();
  const int64_t n = M * row;
  uint4 v[2];
  int64_t at[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int64_t idx = ((int64_t)blockIdx.x * 2 + u) * blockDim.x + threadIdx.x;
    at[u] = -1;
    if (idx < n) {
      const int64_t m = idx / row, j = idx - m * row;
      const uint4* p = src + m * ld_src + j;
      asm volatile("ld.global.cv.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                   : "l"(p)
                   : "memory");
      at[u] = m * ld_dst + j;
    }
  }
  pdl_wait_prior();
#pragma unroll
  for (int u = 0; u < 2; ++u)
    if (at[u] >= 0) dst[at[u]] = v[u];
}

}  // namespace qlin
