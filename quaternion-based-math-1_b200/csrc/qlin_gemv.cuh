// Decode-sized quaternion linear forward on CUDA cores (sm_100a): a
// memory-bound GEMV for at most MT tokens.
//
// Every row warp owns one output quaternion o and walks the whole input
// width: lane l reads the 16-byte pieces W_p[o, 256c + 8l .. +8) of the four
// weight components (128-bit coalesced loads, a warp reads 512 contiguous
// bytes of one row per component and chunk c), so each weight byte crosses
// HBM exactly once and no K split (partials, counters, reduction) is needed.
// All chunks' loads of a row are in flight at once (kGemvDepth chunks of 256
// input quaternions, refilled as each is consumed), issued before the
// dependency wait when the caller declared the weights static.
//
// The Hamilton product of weight quaternion w = (w0, w1, w2, w3) with input
// quaternion x gives all four output components from one set of loads
// (reference quaternion/reference.py:31-45, the 4x4 sign table of
// quaternion/packing.py:18-21):
//   y0 += w0 x0 - w1 x1 - w2 x2 - w3 x3      y1 += w0 x1 + w1 x0 + w2 x3 - w3 x2
//   y2 += w0 x2 - w1 x3 + w2 x0 + w3 x1      y3 += w0 x3 + w1 x2 - w2 x1 + w3 x0
// in fp32, two input quaternions at a time on packed fp32x2 FMAs
// (fma.rn.f32x2: 16 instead of 32 FMA instructions per quaternion pair; the
// multiplies run after the weights land, so their issue count is on the
// call's critical path); the 32 lanes' sums are combined by warp shuffles and
// rounded once with bias and LoRA.  x is staged once per CTA in shared memory
// as fp32, laid out so that a warp's reads are conflict-free and every float4
// read holds two fp32x2 operands (gemv_put_x).  Its rows arrive by bulk copies
// (TMA engine) requested before the weight loads when they are 16-byte
// aligned: by loads, x queued behind the CTA's 64 KB of weight loads and the
// multiplies could only start once the last weights had landed (measured:
// 5.9 -> 5.4 us per call with LoRA).
//
// LoRA (rank <= 32): y += lora_scale * B (A x).  The scaled down projection
// t = lora_scale * A x needs every input, so this call's prologue kernel
// computes it (qlin_prologue_kernel) and this kernel is its programmatic
// dependent: the prologue lets it launch only after waiting for all earlier
// work of the stream, so the row warps read weights and x at once, and one
// more warp per CTA, the LoRA warp, waits for the prologue, reads t and
// publishes it in shared memory at a named barrier that the row warps meet
// only after their weight stream.
#pragma once

#include "qlin_common.cuh"

namespace qlin {

constexpr int kGemvWarps = 8;                // row warps (output quaternions) per CTA
constexpr int kGemvThreads = 32 * kGemvWarps;
constexpr int kGemvLoraThreads = kGemvThreads + 32;  // + the LoRA warp
constexpr int kGemvChunk = 256;              // input quaternions per chunk (8 per lane)
constexpr int kGemvDepth = 4;                // chunks of one row in flight per lane
constexpr int kGemvMaxRank = 32;
constexpr int kGemvMaxTokens = 4;
constexpr int kGemvLoraBar = 1;              // named barrier: row warps + LoRA warp

struct GemvParams {
  const void* x;
  int64_t ld_x;
  const void* w[4];
  int64_t ld_w;
  const void* wq;      // packed weights [N_g][ld_wq][4] (PACKED kernels), else null
  int64_t ld_wq;       // quaternions per packed row (even)
  const void* bias;    // [4*N_g] or null
  const void* lora_a;  // [rank, 4*K_g] or null
  const void* lora_b;  // [4*N_g, rank] or null
  int rank;
  float lora_scale;
  void* y;
  int64_t ld_y;
  int M, K_g, N_g;
  int nch;             // ceil(K_g / kGemvChunk)
  int x_bulk;          // x rows by one bulk copy each (16-byte aligned rows), else by loads
  const void* t;       // LoRA: scaled down projection [M, ld_t] from this call's prologue
  int64_t ld_t;
  int static_weights;  // weights, bias, LoRA A/B not written by earlier work on the stream
  PeerOut peers;       // column-partitioned layer: every output also stored to these
};

// Dynamic shared memory of one CTA: staged x, then (LoRA) t [MT][kGemvMaxRank]
// fp32, then the raw x rows of the bulk copies and their mbarrier.
__host__ __device__ constexpr size_t gemv_smem_bytes(int mt, int nch, bool lora) {
  return (size_t)mt * nch * kGemvChunk * 16 + (lora ? (size_t)mt * kGemvMaxRank * 4 : 0) +
         (size_t)mt * nch * kGemvChunk * 8 + 16;
}

// Eight 16-bit values (16 bytes) -> fp32.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32(h[i]);
}

// Loads of the weights, x, bias, LoRA B and t: L2 only (ld.global.cg) --
// each CTA reads them once, nothing is gained by allocating them in L1 --
// and, through the memory clobber, kept in program order with the
// dependency wait (griddepcontrol.wait, also a memory-clobbering asm).
__device__ __forceinline__ uint4 ld_w_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}
__device__ __forceinline__ uint2 ld_cg_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.cg.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
  return r;
}
__device__ __forceinline__ unsigned short ld_cg_u16(const void* p) {
  unsigned short r;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(r) : "l"(p) : "memory");
  return r;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Staged x (planar weights): for token m, chunk c, lane l and input
// quaternion pair jp (quaternions j = 2jp, 2jp + 1 of the lane's eight
// 256c + 8l + j), two float4 -- A = (x0[j], x0[j+1], x1[j], x1[j+1]) at index
// ((m * nch + c) * 8 + 2jp) * 32 + l and B = (x2[j], x2[j+1], x3[j], x3[j+1])
// 32 float4 further -- so a warp's reads of one (c, jp) are 32 consecutive
// float4 and every read gives the fp32x2 operands of the packed FMAs.
// gemv_put_x stores one quaternion v of input i (chunk c) of token m.
__device__ __forceinline__ void gemv_put_x(float4* xs, int m, int nch, int c, int i, float4 v) {
  const int l = (i / 8) & 31, j = i & 7, e = j & 1;
  float* a = reinterpret_cast<float*>(xs + ((m * nch + c) * 8 + (j & 6)) * 32 + l);
  float* b = a + 32 * 4;
  a[e] = v.x;
  a[2 + e] = v.y;
  b[e] = v.z;
  b[2 + e] = v.w;
}

// Stages x as fp32 quaternions in shared memory (zeros past K_g and past M).
// Item (token m, input quaternion i), numbered m * nq + i: thread tid of
// nthr converts items tid, tid + nthr, ...  (m, i) advance by nthr (at most
// 2 nq) without a division: measured, a division per load delayed the x
// loads by half a microsecond.  issue() requests a batch of 8 items (all its
// loads before any is used), store() converts and stores it.
template <typename T, int MT, bool PACKED>
struct GemvXStager {
  const T* xg;
  int64_t ld_x;
  int M, K_g, nch, nq, nthr, xm, xi;
  float4* xs;
  uint2 raw[8];
  __device__ __forceinline__ GemvXStager(const void* x, int64_t ld, int M_, int K_g_, int nch_, int tid, int nthr_,
                                         float4* xs_)
      : xg(reinterpret_cast<const T*>(x)), ld_x(ld), M(M_), K_g(K_g_), nch(nch_), nq(nch_ * kGemvChunk),
        nthr(nthr_), xm(tid / (nch_ * kGemvChunk)), xi(tid - (tid / (nch_ * kGemvChunk)) * (nch_ * kGemvChunk)),
        xs(xs_) {}
  __device__ __forceinline__ void advance(int& m, int& i) const {
    i += nthr;
    if (i >= nq) { i -= nq; ++m; }
    if (i >= nq) { i -= nq; ++m; }
  }
  __device__ __forceinline__ bool more() const { return xm < MT; }
  __device__ __forceinline__ void issue() {
    int m = xm, i = xi;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      raw[u] = (m < MT && m < M && i < K_g) ? ld_cg_v2(xg + (int64_t)m * ld_x + 4 * (int64_t)i) : make_uint2(0u, 0u);
      advance(m, i);
    }
  }
  __device__ __forceinline__ void store() {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (xm < MT) {
        const T* h = reinterpret_cast<const T*>(&raw[u]);
        const float4 v = make_float4(to_f32(h[0]), to_f32(h[1]), to_f32(h[2]), to_f32(h[3]));
        const int c = xi / kGemvChunk;
        if constexpr (PACKED) {
          // [m][c][parity][128 quaternion pairs]
          const int ic = xi - c * kGemvChunk;
          xs[((xm * nch + c) * 2 + (ic & 1)) * (kGemvChunk / 2) + (ic >> 1)] = v;
        } else {
          gemv_put_x(xs, xm, nch, c, xi, v);
        }
      }
      advance(xm, xi);
    }
  }
};

// One chunk of a row warp's Hamilton products, packed weights: w0..w3[j] are
// components r, i, j, k of this lane's 8 weight quaternions of chunk c; x
// comes from the staged copy ([m][c][parity][128 quaternion pairs]).
template <int MT>
__device__ __forceinline__ void gemv_chunk_fma_packed(float (&acc)[MT][4], const float (&w0)[8], const float (&w1)[8],
                                                      const float (&w2)[8], const float (&w3)[8], const float4* xs,
                                                      int nch, int c, int lane) {
#pragma unroll
  for (int m = 0; m < MT; ++m) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // quaternion 2 (lane + 32 (j / 2)) + (j % 2) of the chunk
      const float4 v = xs[((m * nch + c) * 2 + (j & 1)) * (kGemvChunk / 2) + lane + 32 * (j >> 1)];
      float y0 = acc[m][0], y1 = acc[m][1], y2 = acc[m][2], y3 = acc[m][3];
      y0 = fmaf(w0[j], v.x, y0); y0 = fmaf(-w1[j], v.y, y0); y0 = fmaf(-w2[j], v.z, y0); y0 = fmaf(-w3[j], v.w, y0);
      y1 = fmaf(w0[j], v.y, y1); y1 = fmaf(w1[j], v.x, y1); y1 = fmaf(w2[j], v.w, y1); y1 = fmaf(-w3[j], v.z, y1);
      y2 = fmaf(w0[j], v.z, y2); y2 = fmaf(-w1[j], v.w, y2); y2 = fmaf(w2[j], v.x, y2); y2 = fmaf(w3[j], v.y, y2);
      y3 = fmaf(w0[j], v.w, y3); y3 = fmaf(w1[j], v.z, y3); y3 = fmaf(-w2[j], v.y, y3); y3 = fmaf(w3[j], v.x, y3);
      acc[m][0] = y0; acc[m][1] = y1; acc[m][2] = y2; acc[m][3] = y3;
    }
  }
}

// fp32x2 operands: two fp32 values in one 64-bit register pair.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return make_float2(lo, hi);
}
// d += a * b on both halves (fma.rn.f32x2, sm_100): each half an IEEE fp32 FMA.
__device__ __forceinline__ void f2_fma(uint64_t& d, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}
// Two adjacent 16-bit weights (one 32-bit word, lower address in the low
// half) -> fp32x2.
template <typename T> __device__ __forceinline__ uint64_t w_pair(uint32_t u);
template <> __device__ __forceinline__ uint64_t w_pair<__nv_bfloat16>(uint32_t u) {
  return f2_pack(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
template <> __device__ __forceinline__ uint64_t w_pair<__half>(uint32_t u) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
  return f2_pack(f.x, f.y);
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int k) {
  return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

// One chunk of a row warp's Hamilton products, planar weights: w[p] holds
// component p of this lane's 8 weight quaternions (16-bit, as loaded).  Two
// input quaternions at a time on packed fp32x2 FMAs (half the FMA
// instructions of the scalar form): yp/yn[m][a] collect the positive and
// the negative terms of output component a (at most 2 tokens; above, yp
// takes all terms and yn stays zero), each half one of the two quaternions,
// summed when the row is finished.
template <typename T, int MT>
__device__ __forceinline__ void gemv_chunk_fma2(uint64_t (&yp)[MT][4], uint64_t (&yn)[MT][4], const uint4 (&w)[4],
                                                const float4* xs, int nch, int c, int lane) {
#pragma unroll
  for (int jp = 0; jp < 4; ++jp) {
    const uint32_t u1 = word_of(w[1], jp), u2 = word_of(w[2], jp), u3 = word_of(w[3], jp);
    const uint64_t W0 = w_pair<T>(word_of(w[0], jp)), W1 = w_pair<T>(u1), W2 = w_pair<T>(u2), W3 = w_pair<T>(u3);
    // y0 = w0x0 - w1x1 - w2x2 - w3x3      y1 = w0x1 + w1x0 + w2x3 - w3x2
    // y2 = w0x2 - w1x3 + w2x0 + w3x1      y3 = w0x3 + w1x2 - w2x1 + w3x0
    if constexpr (MT <= 2) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float4 A = xs[((m * nch + c) * 8 + 2 * jp) * 32 + lane];
        const float4 B = xs[((m * nch + c) * 8 + 2 * jp + 1) * 32 + lane];
        const uint64_t X0 = f2_pack(A.x, A.y), X1 = f2_pack(A.z, A.w);
        const uint64_t X2 = f2_pack(B.x, B.y), X3 = f2_pack(B.z, B.w);
        f2_fma(yp[m][0], W0, X0); f2_fma(yn[m][0], W1, X1); f2_fma(yn[m][0], W2, X2); f2_fma(yn[m][0], W3, X3);
        f2_fma(yp[m][1], W0, X1); f2_fma(yp[m][1], W1, X0); f2_fma(yp[m][1], W2, X3); f2_fma(yn[m][1], W3, X2);
        f2_fma(yp[m][2], W0, X2); f2_fma(yn[m][2], W1, X3); f2_fma(yp[m][2], W2, X0); f2_fma(yp[m][2], W3, X1);
        f2_fma(yp[m][3], W0, X3); f2_fma(yp[m][3], W1, X2); f2_fma(yn[m][3], W2, X1); f2_fma(yp[m][3], W3, X0);
      }
    } else {
      // more tokens: the negative terms use negated weight pairs (sign bits of
      // both 16-bit halves flipped), one accumulator pair per component and
      // token, so the accumulators stay within the register budget
      const uint64_t N1 = w_pair<T>(u1 ^ 0x80008000u), N2 = w_pair<T>(u2 ^ 0x80008000u);
      const uint64_t N3 = w_pair<T>(u3 ^ 0x80008000u);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float4 A = xs[((m * nch + c) * 8 + 2 * jp) * 32 + lane];
        const float4 B = xs[((m * nch + c) * 8 + 2 * jp + 1) * 32 + lane];
        const uint64_t X0 = f2_pack(A.x, A.y), X1 = f2_pack(A.z, A.w);
        const uint64_t X2 = f2_pack(B.x, B.y), X3 = f2_pack(B.z, B.w);
        f2_fma(yp[m][0], W0, X0); f2_fma(yp[m][0], N1, X1); f2_fma(yp[m][0], N2, X2); f2_fma(yp[m][0], N3, X3);
        f2_fma(yp[m][1], W0, X1); f2_fma(yp[m][1], W1, X0); f2_fma(yp[m][1], W2, X3); f2_fma(yp[m][1], N3, X2);
        f2_fma(yp[m][2], W0, X2); f2_fma(yp[m][2], N1, X3); f2_fma(yp[m][2], W2, X0); f2_fma(yp[m][2], W3, X1);
        f2_fma(yp[m][3], W0, X3); f2_fma(yp[m][3], W1, X2); f2_fma(yp[m][3], N2, X1); f2_fma(yp[m][3], W3, X0);
      }
    }
  }
}

// After a row warp's last chunk: sum the 32 lanes, add the LoRA up
// projection (lane l takes component l>>3, ranks 4(l&7)..+3 of this row's
// B, braw/lb as loaded; t in shared memory once the named barrier with the
// LoRA warp passes) and the bias, round once and let lane 0 store the
// output quaternion of every token.
template <typename T, int MT, bool LORA, bool PEERS>
__device__ __forceinline__ void gemv_finish(float (&acc)[MT][4], uint2 braw, uint2 lb, const float* tsum, int lane,
                                            bool row_ok, int o, int M, void* y_, int64_t ld_y, const PeerOut& peers) {
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) acc[m][a] += __shfl_xor_sync(0xffffffffu, acc[m][a], s);

  float lora[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int a = 0; a < 4; ++a) lora[m][a] = 0.f;
  if constexpr (LORA) {
    named_bar_sync(kGemvLoraBar, kGemvLoraThreads);  // the LoRA warp has written t
    const T* bh = reinterpret_cast<const T*>(&lb);
    const int lb_r = 4 * (lane & 7);
    float part[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float4 t = *reinterpret_cast<const float4*>(tsum + m * kGemvMaxRank + lb_r);
      float s = to_f32(bh[0]) * t.x;
      s = fmaf(to_f32(bh[1]), t.y, s);
      s = fmaf(to_f32(bh[2]), t.z, s);
      s = fmaf(to_f32(bh[3]), t.w, s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      part[m] = s;  // lanes 8a..8a+7 hold component a (t carries lora_scale)
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int a = 0; a < 4; ++a) lora[m][a] = __shfl_sync(0xffffffffu, part[m], 8 * a);
  }

  if (row_ok && lane == 0) {
    const T* bh = reinterpret_cast<const T*>(&braw);
    float b[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) b[a] = to_f32(bh[a]);
    T* __restrict__ y = reinterpret_cast<T*>(y_);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < M)
        store_out<T, PEERS>(y, peers, (int64_t)m * ld_y + 4 * (int64_t)o,
                            pack4<T>(acc[m][0] + lora[m][0] + b[0], acc[m][1] + lora[m][1] + b[1],
                                     acc[m][2] + lora[m][2] + b[2], acc[m][3] + lora[m][3] + b[3]));
    }
  }
  // Outputs stored to peers are performed at system scope before the CTA
  // ends, so the barrier kernel that follows may signal them.
  if (PEERS) fence_sys();
}

// PACKED: the weights come from one interleaved buffer wq[o][i][p] (the
// packed weight cache; the same layout as x rows): lane l reads 16-byte
// pieces l, l+32, l+64, l+96 of each 256-quaternion chunk of row o -- piece u
// holds all four components of input quaternions 2u and 2u+1, one address
// stream per row instead of four -- and x is staged with even and odd
// quaternions in separate halves so those reads stay conflict-free.
template <typename T, int MT, bool LORA, bool PEERS, bool PACKED = false>
__global__ void __launch_bounds__(kGemvLoraThreads, 1)
qlin_gemv_kernel(const GemvParams prm) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float4* xs = reinterpret_cast<float4*>(smem_raw);
  float* tsum = reinterpret_cast<float*>(smem_raw + (size_t)MT * prm.nch * kGemvChunk * 16);

  // raw x rows (bulk copies) and their mbarrier
  uint8_t* xraw = smem_raw + (size_t)MT * prm.nch * kGemvChunk * 16 + (LORA ? MT * kGemvMaxRank * 4 : 0);
  uint64_t* xbar = reinterpret_cast<uint64_t*>(xraw + (size_t)MT * prm.nch * kGemvChunk * 8);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nthr = blockDim.x;
  const bool lora_warp = LORA && warp == kGemvWarps;
  const int o = blockIdx.x * kGemvWarps + warp;  // this row warp's output quaternion
  const bool row_ok = !lora_warp && o < prm.N_g;
  const int nch = prm.nch;

  if (prm.x_bulk && tid == 0) {
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // ---- row warps: weights, bias, LoRA B ----
  uint4 wv[kGemvDepth][4];
  auto load_chunk = [&](int d, int c) {
    if constexpr (PACKED) {
      const T* row = reinterpret_cast<const T*>(prm.wq) + (int64_t)o * prm.ld_wq * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = c * kGemvChunk + 2 * (lane + 32 * u);  // first of the piece's two quaternions
        wv[d][u] = (row_ok && c < nch && i < prm.K_g) ? ld_w_v4(row + 4 * (int64_t)i) : make_uint4(0u, 0u, 0u, 0u);
      }
    } else {
      const int i = c * kGemvChunk + 8 * lane;
      const bool ok = row_ok && c < nch && i < prm.K_g;
#pragma unroll
      for (int p = 0; p < 4; ++p)
        wv[d][p] = ok ? ld_w_v4(reinterpret_cast<const T*>(prm.w[p]) + (int64_t)o * prm.ld_w + i)
                      : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  uint2 braw = make_uint2(0u, 0u);   // lane 0: bias of the 4 components
  uint2 lb = make_uint2(0u, 0u);     // LoRA B[4o + (lane>>3)][4*(lane&7) .. +4)
  const int lb_r = 4 * (lane & 7);
  auto load_small = [&]() {
    if (row_ok && lane == 0 && prm.bias)
      braw = ld_cg_v2(reinterpret_cast<const T*>(prm.bias) + 4 * (int64_t)o);
    if (LORA && row_ok && lb_r < prm.rank)
      lb = ld_cg_v2(reinterpret_cast<const T*>(prm.lora_b) + (4 * (int64_t)o + (lane >> 3)) * prm.rank + lb_r);
  };
  // Without LoRA this kernel follows the previous kernel of the stream and
  // waits for it before reading what it may have written (weights first when
  // they are static).  With LoRA it follows this call's prologue, whose
  // launch of it implies that all earlier work is complete: no wait before
  // the weights and x, only the LoRA warp waits, for t.
  // x (a few KB) is requested ahead of the weight stream
  GemvXStager<T, MT, PACKED> xst(prm.x, prm.ld_x, prm.M, prm.K_g, nch, tid, nthr, xs);
  if (!LORA && prm.static_weights) {
#pragma unroll
    for (int d = 0; d < kGemvDepth; ++d) load_chunk(d, d);
    load_small();
  }
  if (!LORA) pdl_wait_prior();
  // x by the TMA engine when its rows allow it: one bulk copy per token row,
  // requested before the weight loads and outside the load queue they fill
  if (prm.x_bulk) {
    if (tid == 0) {
      const uint32_t row = (uint32_t)prm.K_g * 8;
      mbar_arrive_expect_tx(xbar, row * (uint32_t)prm.M);
      for (int m = 0; m < prm.M; ++m)
        bulk_load(xraw + (size_t)m * row, reinterpret_cast<const T*>(prm.x) + (int64_t)m * prm.ld_x, row, xbar);
    }
  } else {
    xst.issue();
  }
  if (LORA || !prm.static_weights) {
    if (!lora_warp) {
#pragma unroll
      for (int d = 0; d < kGemvDepth; ++d) load_chunk(d, d);
      load_small();
    }
  }

  // ---- stage x as fp32 quaternions (zeros past K_g and past M) ----
  if (prm.x_bulk) {
    mbar_wait(xbar, 0);
    // two quaternions (16 bytes of raw x) per step; (m, i) advance without a division
    const int nq = nch * kGemvChunk, np = nq / 2;
    int m = tid / np, i = 2 * (tid - (tid / np) * np);
    for (; m < MT;) {
      uint4 r = make_uint4(0u, 0u, 0u, 0u);
      if (m < prm.M && i < prm.K_g) r = *reinterpret_cast<const uint4*>(xraw + ((size_t)m * prm.K_g + i) * 8);
      const T* h = reinterpret_cast<const T*>(&r);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int ie = i + e;
        const float4 v = make_float4(to_f32(h[4 * e]), to_f32(h[4 * e + 1]), to_f32(h[4 * e + 2]), to_f32(h[4 * e + 3]));
        const int c = ie / kGemvChunk;
        if constexpr (PACKED) {
          const int ic = ie - c * kGemvChunk;
          xs[((m * nch + c) * 2 + (ic & 1)) * (kGemvChunk / 2) + (ic >> 1)] = v;
        } else {
          gemv_put_x(xs, m, nch, c, ie, v);
        }
      }
      i += 2 * nthr;
      while (i >= nq) {
        i -= nq;
        ++m;
      }
    }
  } else {
    xst.store();
    while (xst.more()) {
      xst.issue();
      xst.store();
    }
  }
  __syncthreads();

  if constexpr (LORA) {
    if (lora_warp) {
      // ---------------- LoRA warp ----------------
      pdl_wait_prior();  // the prologue's t is complete
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float v = 0.f;
        if (m < prm.M && lane < prm.rank) {
          const unsigned short h = ld_cg_u16(reinterpret_cast<const T*>(prm.t) + m * prm.ld_t + lane);
          v = to_f32(*reinterpret_cast<const T*>(&h));
        }
        tsum[m * kGemvMaxRank + lane] = v;
      }
      __syncwarp();
      named_bar_arrive(kGemvLoraBar, kGemvLoraThreads);  // t is in shared memory
      return;
    }
  }

  // ---- row warps: the Hamilton product over all input quaternions ----
  float acc[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int a = 0; a < 4; ++a) acc[m][a] = 0.f;
  if constexpr (!PACKED) {
    uint64_t yp[MT][4], yn[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int a = 0; a < 4; ++a) yp[m][a] = yn[m][a] = 0ull;
    for (int cb = 0; cb < nch; cb += kGemvDepth) {
#pragma unroll
      for (int d = 0; d < kGemvDepth; ++d) {
        const int c = cb + d;
        if (c < nch) {
          const uint4 w[4] = {wv[d][0], wv[d][1], wv[d][2], wv[d][3]};
          // refill: the chunk kGemvDepth further on reuses these registers
          if (c + kGemvDepth < nch) load_chunk(d, c + kGemvDepth);
          gemv_chunk_fma2<T, MT>(yp, yn, w, xs, nch, c, lane);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float2 p = f2_unpack(yp[m][a]), n = f2_unpack(yn[m][a]);
        acc[m][a] = (p.x + p.y) - (n.x + n.y);
      }
  }
  for (int cb = 0; PACKED && cb < nch; cb += kGemvDepth) {
#pragma unroll
    for (int d = 0; d < kGemvDepth; ++d) {
      const int c = cb + d;
      if (c < nch) {
        // w0..w3[j]: components r, i, j, k of this lane's 8 weight quaternions
        float w0[8], w1[8], w2[8], w3[8];
        // piece u holds quaternions 2u' and 2u'+1 (u' = lane + 32u) as r,i,j,k,r,i,j,k
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float f[8];
          unpack8<T>(wv[d][u], f);
          w0[2 * u] = f[0]; w1[2 * u] = f[1]; w2[2 * u] = f[2]; w3[2 * u] = f[3];
          w0[2 * u + 1] = f[4]; w1[2 * u + 1] = f[5]; w2[2 * u + 1] = f[6]; w3[2 * u + 1] = f[7];
        }
        // refill: the chunk kGemvDepth further on reuses these registers
        if (c + kGemvDepth < nch) load_chunk(d, c + kGemvDepth);
        gemv_chunk_fma_packed<MT>(acc, w0, w1, w2, w3, xs, nch, c, lane);
      }
    }
  }
  gemv_finish<T, MT, LORA, PEERS>(acc, braw, lb, tsum, lane, row_ok, o, prm.M, prm.y, prm.ld_y, prm.peers);
}

}  // namespace qlin
