// C ABI of the B200 quaternion linear forward (declarations: include/qlin_b200.h).
//
// Host responsibilities: argument validation with the reference's error
// classes (shape -> QLIN_ERR_SHAPE, which the Python layer raises as
// ValueError like quaternion/packing.py:45-52 and quaternion/linear.py:55-61),
// kernel selection, workspace carving, TMA descriptor encoding and launch on
// the caller's stream.  No exception crosses the ABI, nothing allocates.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>  // types only: the functions are resolved at run time

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "../../include/qlin_b200.h"
#include "qlin_gemv.cuh"
#include "qlin_simt.cuh"
#include "qlin_pair.cuh"
#include "qlin_tc.cuh"

namespace {

using namespace qlin;

constexpr int kMaxDevices = 64;

// The packed weight cache of a call: wq[o][i][p] (all four components of a
// weight quaternion side by side, the layout of x), ld in quaternions; null
// when the call has planar weights only.
struct PackedW {
  const void* w = nullptr;
  int64_t ld = 0;
};

struct DeviceInfo {
  bool init = false;
  int cc_major = 0, cc_minor = 0, num_sms = 0;
  // per (element type, N_TOK, in-kernel LoRA) kernel instance: attributes
  // set, and how many CTAs of it the device keeps resident at once
  bool tc_attr_set[2][4][3][2][2] = {};  // [dtype][N_TOK][LoRA mode][peers][cluster]
  int resident[2][4][3][2][2] = {};
  // cluster K split: how many clusters of `split` CTAs fit at once, by
  // [dtype][LoRA mode][split] (-1: not queried yet)
  int cluster_cap[2][3][kTcClusterMax + 1];
  // CUDA-core decode kernel: shared-memory limit raised, by [dtype][MT][LoRA][peers]
  bool gemv_attr_set[2][3][2][2][2] = {};  // [dtype][MT][LoRA][peers][packed]
  // CTA-pair prefill kernel: attributes set and how many pairs fit at once, by [dtype][peers][tile]
  bool pair_attr_set[2][2][2][2] = {};  // [dtype][peers][tile][packed]
  int pair_cap[2][2][2][2] = {};
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_mutex;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int device_info(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QLIN_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceInfo& d = g_dev[dev];
  if (!d.init) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return QLIN_ERR_LAUNCH;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.num_sms = prop.multiProcessorCount;
    for (auto& a : d.cluster_cap)
      for (auto& b : a)
        for (int& c : b) c = -1;
    d.init = true;
  }
  *out = &d;
  return (d.cc_major == 10) ? QLIN_OK : QLIN_ERR_DEVICE;
}

int get_encoder() {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_encode) return QLIN_OK;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn)
    return QLIN_ERR_LAUNCH;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return QLIN_OK;
}

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline size_t elem_size(int dtype) { return dtype == QLIN_F32 ? 4 : 2; }

// Tokens up to which the tensor-core path builds its activation operand in
// shared memory (stacked mode) instead of reading component planes.
constexpr int64_t kStackMaxTokens = 64;

// Upper bound of the SM count of an sm_100 part, used to size the split-K
// partials before a device is known.
constexpr int64_t kMaxSms = 160;

int n_tok_for(int64_t M) { return M <= 16 ? 16 : (M <= 32 ? 32 : (M <= kStackMaxTokens ? 64 : 128)); }
int n_tok_index(int n_tok) { return n_tok == 16 ? 0 : (n_tok == 32 ? 1 : (n_tok == 64 ? 2 : 3)); }

// Largest K split the tensor-core path uses for this problem on a device with
// `sms` SMs: all CTAs of all splits of all tiles fit in one wave, every CTA
// keeps at least one K chunk, at most kTcMaxSplit; no split when the tiles
// alone fill half the device.
int max_split_for(int64_t M, int64_t K_g, int64_t N_g, int64_t sms) {
  const int64_t n_tok = n_tok_for(M);
  const int64_t tiles = ((N_g + kTcBlockO - 1) / kTcBlockO) * ((M + n_tok - 1) / n_tok);
  const int64_t chunks = (K_g + kTcChunk - 1) / kTcChunk;
  if (tiles == 0 || tiles * 2 > sms) return 1;
  const int64_t s = std::min<int64_t>({(int64_t)kTcMaxSplit, chunks, std::max<int64_t>(1, sms / tiles)});
  return (int)std::max<int64_t>(1, s);
}

// Workspace pieces.  Tensor-core path: planar x (4 * M * K_g 16-bit, M > 64),
// scaled LoRA t ([M, round_up(rank, 8)] 16-bit), split-K partials (fp32 x4 per
// split, tile, token and row).  CUDA-core path: LoRA t ([M, rank] fp32).
struct WsLayout {
  size_t xp_off = 0, xp_bytes = 0, t_off = 0, t_bytes = 0, tf_off = 0, tf_bytes = 0;
  size_t part_off = 0, part_bytes = 0, cnt_off = 0, cnt_bytes = 0, total = 0;
  int64_t ld_t = 0;
};

// Tokens up to which a K split sums its partials inside the main kernel (the
// last CTA of each tile to arrive reads every slot); above, a separate
// reduction kernel spreads that work over the device.
constexpr int64_t kFusedReduceMaxTokens = 4;

// K split of the fp32 CUDA-core kernel (qlin_simt_splitk_kernel): enough CTAs
// of 64 tokens x 32 output quaternions to cover the SMs, each split keeping at
// least one 8-quaternion step, at most 8; none when the tiles alone cover
// half the SMs.
int f32_split_for(int64_t M, int64_t K_g, int64_t N_g, int64_t sms) {
  const int64_t tiles = ((M + kSkBM - 1) / kSkBM) * ((N_g + kSkBO - 1) / kSkBO);
  const int64_t steps = (K_g + kSkBK - 1) / kSkBK;
  if (tiles == 0 || tiles * 2 > sms) return 1;
  return (int)std::max<int64_t>(1, std::min<int64_t>({8, steps, sms / tiles}));
}

WsLayout ws_layout(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank) {
  WsLayout w;
  // The first QLIN_WORKSPACE_COUNTER_BYTES of every non-empty workspace are
  // the arrival counters of the fused split-K reduction (used only under
  // QLIN_FLAG_ZEROED_WORKSPACE); nothing else is ever placed there.
  w.cnt_off = 0;
  w.cnt_bytes = QLIN_WORKSPACE_COUNTER_BYTES;
  size_t off = w.cnt_bytes;
  if (dtype != QLIN_F32) {
    w.xp_off = off;
    w.xp_bytes = M > kStackMaxTokens ? (size_t)(4 * M * K_g * 2) : 0;
    off = (size_t)round_up((int64_t)(off + w.xp_bytes), 256);
    if (rank > 0) {
      w.ld_t = round_up(rank, 8);
      w.t_off = off;
      w.t_bytes = (size_t)(M * w.ld_t * 2);
      off = (size_t)round_up((int64_t)(off + w.t_bytes), 256);
    }
    const int split = max_split_for(M, K_g, N_g, kMaxSms);
    if (split > 1) {
      const int64_t n_tok = n_tok_for(M);
      const int64_t tiles = ((N_g + kTcBlockO - 1) / kTcBlockO) * ((M + n_tok - 1) / n_tok);
      w.part_off = off;
      w.part_bytes = (size_t)(split * tiles * n_tok * kTcBlockO * 16);
      off = (size_t)round_up((int64_t)(off + w.part_bytes), 256);
    }
  }
  if (rank > 0) {
    w.tf_off = off;
    w.tf_bytes = (size_t)(M * rank * 4);
    off = (size_t)round_up((int64_t)(off + w.tf_bytes), 256);
  }
  if (dtype == QLIN_F32) {
    // fp32 partials of the K split [split][M][4 N_g]
    const int split = f32_split_for(M, K_g, N_g, kMaxSms);
    if (split > 1) {
      w.part_off = off;
      w.part_bytes = (size_t)(split * M * 4 * N_g * 4);
      off = (size_t)round_up((int64_t)(off + w.part_bytes), 256);
    }
  }
  // A problem that needs no scratch needs no counters either.
  w.total = (M == 0 || off == w.cnt_bytes) ? 0 : off;
  return w;
}

int validate(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi, const void* wj,
             const void* wk, int64_t ld_w, const void* lora_a, const void* lora_b, int rank,
             const void* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g, const PackedW* pw = nullptr) {
  const bool planar = wr || wi || wj || wk;
  const bool packed = pw && pw->w;
  if (dtype != QLIN_F32 && dtype != QLIN_BF16 && dtype != QLIN_F16) return QLIN_ERR_DTYPE;
  if (M < 0 || K_g <= 0 || N_g <= 0 || rank < 0) return QLIN_ERR_SHAPE;
  if (ld_x < 4 * K_g || (planar && ld_w < K_g) || ld_y < 4 * N_g) return QLIN_ERR_SHAPE;
  if (packed && pw->ld < K_g) return QLIN_ERR_SHAPE;
  if (M > INT32_MAX || N_g > INT32_MAX / 4 || K_g > INT32_MAX / 4) return QLIN_ERR_SHAPE;
  if (M == 0) return QLIN_OK;
  if (!x || !y || !(packed || planar)) return QLIN_ERR_ARG;
  if (planar && (!wr || !wi || !wj || !wk)) return QLIN_ERR_ARG;
  if (rank > 0 && (!lora_a || !lora_b)) return QLIN_ERR_ARG;
  return QLIN_OK;
}

bool tc_eligible(int dtype, const void* x, int64_t ld_x, const void* const w[4], int64_t ld_w,
                 const void* lora_a, const void* lora_b, int rank, const void* y, int64_t ld_y,
                 int64_t K_g) {
  if (dtype == QLIN_F32) return false;
  if (K_g % 8 != 0 || ld_x % 8 != 0 || ld_w % 8 != 0 || ld_y % 4 != 0) return false;
  if (!aligned(x, 16) || !aligned(y, 8)) return false;
  for (int p = 0; p < 4; ++p)
    if (!aligned(w[p], 16)) return false;
  if (rank > 0 && (rank % 8 != 0 || !aligned(lora_b, 16) || !aligned(lora_a, 16))) return false;
  return true;
}

int select_algo(int dtype) { return dtype == QLIN_F32 ? QLIN_ALGO_SIMT : QLIN_ALGO_TC; }

// Tokens up to which QLIN_ALGO_AUTO runs the CUDA-core decode kernel (when
// eligible) instead of the tensor-core kernel.
constexpr int64_t kGemvAutoTokens = 2;
// Largest LoRA rank for which QLIN_ALGO_AUTO runs the decode kernel.
constexpr int kGemvAutoRank = 32;

// Largest shared memory the decode kernel may ask for (staged x + LoRA slots).
constexpr size_t kGemvMaxSmem = 200 * 1024;

int gemv_tokens(int64_t M) { return M <= 1 ? 1 : (M <= 2 ? 2 : 4); }

// QLIN_ALGO_AUTO's choice of the decode kernel: at most kGemvAutoTokens
// tokens and output quaternions for at most one CTA of 8 warps per SM (one
// wave: every CTA's latency-bound start and end then overlap the others'
// weight streams; larger layers keep the pipelined tensor-core kernel).
bool gemv_auto(int64_t M, int64_t N_g, int rank, const DeviceInfo* dev) {
  return M <= kGemvAutoTokens && rank <= kGemvAutoRank && (N_g + kGemvWarps - 1) / kGemvWarps <= dev->num_sms;
}

// The CUDA-core decode kernel: 16-bit types, at most kGemvMaxTokens tokens,
// 16-byte weight pieces (K_g and ld_w multiples of 8, 16-byte aligned
// weights), 8-byte x quaternions, bias and output stores, LoRA rank at most
// 32 and a multiple of 4, staged x within kGemvMaxSmem.
bool gemv_eligible(int dtype, const void* x, int64_t ld_x, const void* const w[4], int64_t ld_w,
                   const void* bias, const void* lora_a, const void* lora_b, int rank, const void* y,
                   int64_t ld_y, int64_t M, int64_t K_g) {
  if (dtype == QLIN_F32 || M > kGemvMaxTokens) return false;
  if (K_g % 8 != 0 || ld_w % 8 != 0 || ld_x % 4 != 0 || ld_y % 4 != 0) return false;
  if (!aligned(x, 8) || !aligned(y, 8) || (bias && !aligned(bias, 8))) return false;
  for (int p = 0; p < 4; ++p)
    if (!aligned(w[p], 16)) return false;
  // LoRA: the prologue kernel reads x and lora_a in 16-byte vectors
  if (rank > 0 && (rank > kGemvMaxRank || rank % 4 != 0 || !aligned(lora_a, 16) || !aligned(lora_b, 8) ||
                   !aligned(x, 16) || ld_x % 8 != 0))
    return false;
  const int nch = (int)((K_g + kGemvChunk - 1) / kGemvChunk);
  return gemv_smem_bytes(gemv_tokens(M), nch, rank > 0) <= kGemvMaxSmem;
}

CUresult encode(CUtensorMap* map, CUtensorMapDataType dt, int rank, void* base, const cuuint64_t* dims,
                const cuuint64_t* strides, const cuuint32_t* box,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_64B) {
  cuuint32_t estr[3] = {1, 1, 1};
  return g_encode(map, dt, (cuuint32_t)rank, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// Stacked activation operand for N_TOK <= 64 (decode-sized M), planes above.
template <int N_TOK>
constexpr bool kStackFor = N_TOK <= kStackMaxTokens;

// Where the LoRA down projection runs (kLora*), for ranks up to
// kTcLoraInRank: on the builder warps' CUDA cores for at most
// kTcLoraSimtTokens tokens when each split covers at most 4 K chunks (a few
// hundred multiply-adds per thread, hidden under the weight stream); on the
// tensor cores inside the main kernel for stacked tiles of at most 32 tokens
// (their TMEM lanes 64..95 belong to builder warp 2); else in the prologue.
int lora_mode(int64_t M, int rank, int64_t K_g, int split) {
  if (rank <= 0 || rank > kTcLoraInRank) return kLoraPrologue;
  const int64_t chunks = (K_g + kTcChunk - 1) / kTcChunk;
  if (M <= kTcLoraSimtTokens && (chunks + split - 1) / split <= 4) return kLoraSimt;
  if (n_tok_for(M) <= 32) return kLoraTc;
  return kLoraPrologue;
}

// Threads of a tensor-core CTA: 128, plus two LoRA warps in the CUDA-core mode.
constexpr int tc_block_threads(int lora) { return lora == kLoraSimt ? kTcMaxThreads : kTcThreads; }

// K split the device path uses (same-box measurements on B200, 4096-wide
// decode layer).  At most 2 tokens: 8 splits, one cluster per tile, summed
// through distributed shared memory (6.6 vs 8.1 us/call with LoRA r=32, 6.2
// vs 6.8 without) -- except with static weights and no LoRA, where 16
// splits prefetching their weights stay faster (5.9 vs 6.3).  With the
// CUDA-core LoRA (at most 4 tokens) every split also loads LoRA B and
// applies its own LoRA term, a fixed cost per CTA: at most 8 splits there.
int split_for(int64_t M, int64_t K_g, int64_t N_g, int rank, int64_t sms, bool static_weights = false) {
  const int s = max_split_for(M, K_g, N_g, sms);
  const int64_t chunks = (K_g + kTcChunk - 1) / kTcChunk;
  if (M <= 2 && s > 8 && !(static_weights && rank == 0)) return 8;
  if (rank > 0 && rank <= kTcLoraInRank && M <= kTcLoraSimtTokens && s > 8 && (chunks + 7) / 8 <= 4) return 8;
  return s;
}

template <typename T, int N_TOK, int LORA, bool PEERS = false, bool CLUSTER = false>
int ensure_tc_attrs(DeviceInfo* dev) {
  using Cfg = TcCfg<N_TOK, kStackFor<N_TOK>, LORA, CLUSTER>;
  auto kernel = qlin_tc_kernel<T, N_TOK, kStackFor<N_TOK>, LORA, PEERS, CLUSTER>;
  const int ti = n_tok_index(N_TOK);
  const int di = std::is_same<T, __nv_bfloat16>::value ? 0 : 1;
  const int li = LORA, pi = PEERS ? 1 : 0, ci = CLUSTER ? 1 : 0;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (dev->tc_attr_set[di][ti][li][pi][ci]) return QLIN_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) !=
      cudaSuccess)
    return QLIN_ERR_LAUNCH;
  // clusters of up to 16 CTAs (the cluster K split of decode tiles)
  if (CLUSTER && cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return QLIN_ERR_LAUNCH;
  // Every kernel of the call prefers the full shared-memory carveout, so the
  // SMs need no L1/shared reconfiguration between the prologue, the main
  // kernel and the split-K reduction.
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
      cudaFuncSetAttribute(qlin_splitk_reduce_kernel<T>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
      cudaFuncSetAttribute(qlin_prologue_kernel<T, 1>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
      cudaFuncSetAttribute(qlin_prologue_kernel<T, 8>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return QLIN_ERR_LAUNCH;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, tc_block_threads(LORA), Cfg::kSmemBytes) !=
      cudaSuccess)
    return QLIN_ERR_LAUNCH;
  dev->resident[di][ti][li][pi][ci] = per_sm * dev->num_sms;
  dev->tc_attr_set[di][ti][li][pi][ci] = true;
  return QLIN_OK;
}

// Whether every cluster of a decode grid (tiles clusters of `split` CTAs, the
// cluster K split) fits on the device at once.
template <typename T, int LORA>
bool cluster_fits(DeviceInfo* dev, int split, int64_t tiles) {
  if (split < 2 || split > kTcClusterMax) return false;
  {
    const int di = std::is_same<T, __nv_bfloat16>::value ? 0 : 1;
    int cap;
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      cap = dev->cluster_cap[di][LORA][split];
    }
    if (cap < 0) {
      if (ensure_tc_attrs<T, 16, LORA, false, true>(dev) != QLIN_OK) return false;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)split, (unsigned)tiles, 1);
      cfg.blockDim = dim3(tc_block_threads(LORA), 1, 1);
      cfg.dynamicSmemBytes = TcCfg<16, true, LORA, true>::kSmemBytes;
      cudaLaunchAttribute a;
      a.id = cudaLaunchAttributeClusterDimension;
      a.val.clusterDim.x = (unsigned)split;
      a.val.clusterDim.y = 1;
      a.val.clusterDim.z = 1;
      cfg.attrs = &a;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, qlin_tc_kernel<T, 16, true, LORA, false, true>, &cfg) != cudaSuccess)
        n = 0;
      cudaGetLastError();
      cap = n;
      std::lock_guard<std::mutex> lock(g_mutex);
      dev->cluster_cap[di][LORA][split] = cap;
    }
    return cap >= tiles;
  }
}

// The cluster K split a decode-sized problem uses (0: none): at most
// kTcClusterTokens tokens (tiles of 16), the K split split_for chose (at most
// 8 for one or two tokens: with static weights and no LoRA the 16 plain
// splits, prefetching their weights, measured faster), when all clusters of
// the grid fit at once; else 8 CTAs per cluster when that fits (and keeps
// the CUDA-core LoRA mode's slice of at most 4 chunks per split).  Same-box
// measurements, 4096 layer with bias and LoRA r=32 (x rows by TMA): 4, 8, 16
// tokens 9.95, 9.32, 10.46 us/call in 8-CTA clusters (one launch) against
// 11.75, 10.44, 10.56 through the workspace (16-CTA clusters do not all fit
// at once on this part).
template <typename T, int LORA>
int cluster_split(DeviceInfo* dev, int64_t M, int64_t K_g, int split, int64_t tiles) {
  if (M > kTcClusterTokens || split < 2 || (M <= 2 && split > 8)) return 0;
  // every owner's receive slots, (C - 1) * ceil(M / C), fit the buffer
  auto slots_ok = [&](int c) { return (c - 1) * ((M + c - 1) / c) <= kTcClusterSlots; };
  if (slots_ok(split) && cluster_fits<T, LORA>(dev, split, tiles)) return split;
  const int64_t chunks = (K_g + kTcChunk - 1) / kTcChunk;
  if (split > 8 && M <= 16 && slots_ok(8) && (LORA != kLoraSimt || (chunks + 7) / 8 <= 4) &&
      cluster_fits<T, LORA>(dev, 8, tiles))
    return 8;
  return 0;
}

template <typename T, int N_TOK, int LORA>
int launch_tc_impl(DeviceInfo* dev, const CUtensorMap* maps, const TcParams& base_prm, int64_t M,
                   int64_t K_g, int64_t N_g, float4* partials, cudaStream_t stream) {
  using Cfg = TcCfg<N_TOK, kStackFor<N_TOK>, LORA>;
  // outputs also stored to peers only in the column-partitioned path's build
  const bool peers = has_peers(base_prm.peers);
  {
    const int64_t o_blocks = (N_g + kTcBlockO - 1) / kTcBlockO, t_blocks = (M + N_TOK - 1) / N_TOK;
    const int split = split_for(M, K_g, N_g, base_prm.rank, dev->num_sms, base_prm.static_weights != 0);
    if constexpr (N_TOK == 16) {
      const int cs = (peers || base_prm.no_cluster) ? 0 : cluster_split<T, LORA>(dev, M, K_g, split, o_blocks * t_blocks);
      if (cs > 0) {
        TcParams prm = base_prm;
        prm.split_k = cs;
        prm.partials = nullptr;
        prm.fuse_reduce = 0;
        cudaLaunchAttribute attrs[2];
        attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[0].val.programmaticStreamSerializationAllowed = 1;
        attrs[1].id = cudaLaunchAttributeClusterDimension;
        attrs[1].val.clusterDim.x = (unsigned)cs;
        attrs[1].val.clusterDim.y = 1;
        attrs[1].val.clusterDim.z = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)cs, (unsigned)o_blocks, (unsigned)t_blocks);
        cfg.blockDim = dim3(tc_block_threads(LORA), 1, 1);
        cfg.dynamicSmemBytes = TcCfg<16, true, LORA, true>::kSmemBytes;
        cfg.stream = stream;
        cfg.attrs = attrs;
        cfg.numAttrs = 2;
        return cudaLaunchKernelEx(&cfg, qlin_tc_kernel<T, 16, true, LORA, false, true>, maps[0], maps[1],
                                  maps[2], maps[3], maps[4], maps[5], maps[6], maps[7], prm) == cudaSuccess
                   ? QLIN_OK
                   : QLIN_ERR_LAUNCH;
      }
    }
  }
  auto kernel = peers ? qlin_tc_kernel<T, N_TOK, kStackFor<N_TOK>, LORA, true>
                      : qlin_tc_kernel<T, N_TOK, kStackFor<N_TOK>, LORA, false>;
  int st = peers ? ensure_tc_attrs<T, N_TOK, LORA, true>(dev) : ensure_tc_attrs<T, N_TOK, LORA, false>(dev);
  if (st != QLIN_OK) return st;
  TcParams prm = base_prm;
  const int64_t o_blocks = (N_g + kTcBlockO - 1) / kTcBlockO;
  const int64_t t_blocks = (M + N_TOK - 1) / N_TOK;
  if (o_blocks > 65535 || t_blocks > 65535) return QLIN_ERR_SHAPE;
  const int split = split_for(M, K_g, N_g, base_prm.rank, dev->num_sms, base_prm.static_weights != 0);
  prm.split_k = split;
  prm.partials = split > 1 ? partials : nullptr;
  if (split > 1 && !partials) return QLIN_ERR_WORKSPACE;
  prm.fuse_reduce = (split > 1 && M <= kFusedReduceMaxTokens && prm.counters) ? 1 : 0;
  // one counter per output tile, all inside the counter bytes
  if (prm.fuse_reduce && o_blocks * t_blocks * 4 > (int64_t)QLIN_WORKSPACE_COUNTER_BYTES) prm.fuse_reduce = 0;

  // Programmatic dependent launch: the kernel's set-up overlaps the tail of
  // the previous kernel of the stream; it waits for that kernel
  // (griddepcontrol.wait) before touching memory.
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)split, (unsigned)o_blocks, (unsigned)t_blocks);
  cfg.blockDim = dim3(tc_block_threads(LORA), 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, maps[0], maps[1], maps[2], maps[3], maps[4],
                                     maps[5], maps[6], maps[7], prm);
  if (e != cudaSuccess) return QLIN_ERR_LAUNCH;
  if (split > 1 && !prm.fuse_reduce) {
    // The reduction is a programmatic dependent of the main kernel, which
    // lets it launch at once; it waits for the main grid before reading.
    const int64_t threads = t_blocks * o_blocks * N_TOK * kTcBlockO;
    cudaLaunchConfig_t rc = {};
    rc.gridDim = dim3((unsigned)((threads + 255) / 256), 1, 1);
    rc.blockDim = dim3(256, 1, 1);
    rc.stream = stream;
    rc.attrs = &attr;
    rc.numAttrs = 1;
    e = cudaLaunchKernelEx(&rc, qlin_splitk_reduce_kernel<T>, (const float4*)partials, split,
                           (int)t_blocks, (int)o_blocks, N_TOK, static_cast<const T*>(prm.bias),
                           static_cast<T*>(prm.y), prm.ld_y, prm.M, prm.N_g, prm.static_weights, prm.peers);
    if (e != cudaSuccess) return QLIN_ERR_LAUNCH;
  }
  return QLIN_OK;
}

// The CTA-pair kernel (qlin_pair.cuh) takes prefill-sized problems without
// LoRA: more than kStackMaxTokens tokens, 16-byte output pieces (ld_y a
// multiple of 8, 16-byte aligned y and peer outputs, an even number of
// output quaternions) on top of the tensor-core path's TMA rules.
bool pair_eligible(int64_t M, int64_t N_g, int rank, const void* y, int64_t ld_y, const PeerOut& peers,
                   int flags) {
  if (M <= kStackMaxTokens || rank != 0 || (flags & QLIN_FLAG_NO_PAIR) || N_g % 2 != 0 || ld_y % 8 != 0 ||
      !aligned(y, 16))
    return false;
  for (int p = 0; p < peers.n; ++p)
    if (!aligned(peers.y[p], 16)) return false;
  return !peers.mc || aligned(peers.mc, 16);
}

template <typename T, bool PEERS, int NTOK, bool PACKED = false>
int pair_attrs(DeviceInfo* dev, int* cap) {
  const int di = std::is_same<T, __nv_bfloat16>::value ? 0 : 1;
  const int pi = PEERS ? 1 : 0, ti = NTOK == 256 ? 1 : 0, ki = PACKED ? 1 : 0;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!dev->pair_attr_set[di][pi][ti][ki]) {
    auto kernel = qlin_pair_kernel<T, PEERS, NTOK, PACKED>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes) != cudaSuccess)
      return QLIN_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = kPairSmemBytes;
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeClusterDimension;
    a.val.clusterDim.x = 2;
    a.val.clusterDim.y = 1;
    a.val.clusterDim.z = 1;
    cfg.attrs = &a;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return QLIN_ERR_LAUNCH;
    }
    dev->pair_cap[di][pi][ti][ki] = n;
    dev->pair_attr_set[di][pi][ti][ki] = true;
  }
  *cap = dev->pair_cap[di][pi][ti][ki];
  return QLIN_OK;
}

// Tokens per tile of the CTA-pair kernel: 256 (one accumulator, 128 cycles
// per UMMA) above 128 tokens, else 128.
inline int pair_tokens(int64_t M) { return M > 128 ? 256 : 128; }

// Tiles of the CTA-pair kernel: 256 real outputs x pair_tokens(M) tokens.
inline int64_t pair_tiles(int64_t M, int64_t N_g) {
  const int64_t nt = pair_tokens(M);
  return ((4 * N_g + 255) / 256) * ((M + nt - 1) / nt);
}

template <typename T, bool PEERS, int NTOK, bool PACKED>
int launch_pair(DeviceInfo* dev, const T* x, int64_t ld_x, const void* const w[4], int64_t ld_w,
                const PackedW& pw, const T* bias, T* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g,
                const PeerOut& peers, cudaStream_t stream) {
  int cap = 0;
  int st = pair_attrs<T, PEERS, NTOK, PACKED>(dev, &cap);
  if (st != QLIN_OK) return st;
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // x [M, 4*K_g]: 64-element x NTOK/2-token boxes, 128-byte swizzle (the UMMA
  // B operand); W_p [N_g, K_g]: 32-element x 32-row boxes, 64-byte swizzle
  // (read by the builder warps).  Out-of-range rows and columns read as zero.
  CUtensorMap maps[5];
  std::memset(maps, 0, sizeof(maps));
  {
    cuuint64_t dims[2] = {(cuuint64_t)(4 * K_g), (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)(ld_x * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)PairCfg<NTOK>::kHalf};
    if (encode(&maps[0], dt, 2, const_cast<T*>(x), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return QLIN_ERR_ALIGN;
  }
  if (PACKED) {
    // wq [N_g][ld][4]: 64-element (16-quaternion) x 32-row boxes, 128-byte swizzle
    cuuint64_t dims[2] = {(cuuint64_t)(4 * K_g), (cuuint64_t)N_g};
    cuuint64_t strides[1] = {(cuuint64_t)(pw.ld * 8)};
    cuuint32_t box[2] = {64, 32};
    if (encode(&maps[1], dt, 2, const_cast<void*>(pw.w), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) !=
        CUDA_SUCCESS)
      return QLIN_ERR_ALIGN;
  } else {
    for (int p = 0; p < 4; ++p) {
      cuuint64_t dims[2] = {(cuuint64_t)K_g, (cuuint64_t)N_g};
      cuuint64_t strides[1] = {(cuuint64_t)(ld_w * 2)};
      cuuint32_t box[2] = {32, 32};
      if (encode(&maps[1 + p], dt, 2, const_cast<void*>(w[p]), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B) !=
          CUDA_SUCCESS)
        return QLIN_ERR_ALIGN;
    }
  }
  const int64_t tiles = pair_tiles(M, N_g);
  if (tiles > INT32_MAX) return QLIN_ERR_SHAPE;
  PairParams prm{};
  prm.bias = bias;
  prm.y = y;
  prm.ld_y = ld_y;
  prm.M = (int)M;
  prm.N_g = (int)N_g;
  prm.K_g = (int)K_g;
  prm.stages = (int)((K_g + 31) / 32);
  prm.nb_tiles = (int)((4 * N_g + 255) / 256);
  prm.tiles = (int)tiles;
  prm.peers = peers;
  const int64_t pairs = std::min<int64_t>(tiles, cap);
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  attrs[1].id = cudaLaunchAttributeClusterDimension;
  attrs[1].val.clusterDim.x = 2;
  attrs[1].val.clusterDim.y = 1;
  attrs[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, qlin_pair_kernel<T, PEERS, NTOK, PACKED>, maps[0], maps[1], maps[2], maps[3], maps[4],
                            prm) == cudaSuccess
             ? QLIN_OK
             : QLIN_ERR_LAUNCH;
}

// Peer outputs (column-partitioned layer) get the kernel variant that also
// stores every output piece into them.
template <typename T, bool PEERS>
int run_pair_p(DeviceInfo* dev, const T* x, int64_t ld_x, const void* const w[4], int64_t ld_w, const PackedW& pw,
               const T* bias, T* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g, const PeerOut& peers,
               cudaStream_t stream) {
  const bool big = pair_tokens(M) == 256;
  if (pw.w)
    return big ? launch_pair<T, PEERS, 256, true>(dev, x, ld_x, w, ld_w, pw, bias, y, ld_y, M, K_g, N_g, peers, stream)
               : launch_pair<T, PEERS, 128, true>(dev, x, ld_x, w, ld_w, pw, bias, y, ld_y, M, K_g, N_g, peers, stream);
  return big ? launch_pair<T, PEERS, 256, false>(dev, x, ld_x, w, ld_w, pw, bias, y, ld_y, M, K_g, N_g, peers, stream)
             : launch_pair<T, PEERS, 128, false>(dev, x, ld_x, w, ld_w, pw, bias, y, ld_y, M, K_g, N_g, peers, stream);
}

template <typename T>
int run_pair(DeviceInfo* dev, const T* x, int64_t ld_x, const void* const w[4], int64_t ld_w, const PackedW& pw,
             const T* bias, T* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g, const PeerOut& peers,
             cudaStream_t stream) {
  if (get_encoder() != QLIN_OK) return QLIN_ERR_LAUNCH;
  if (has_peers(peers)) return run_pair_p<T, true>(dev, x, ld_x, w, ld_w, pw, bias, y, ld_y, M, K_g, N_g, peers, stream);
  return run_pair_p<T, false>(dev, x, ld_x, w, ld_w, pw, bias, y, ld_y, M, K_g, N_g, peers, stream);
}

template <typename T>
int run_tc(DeviceInfo* dev, const T* x, int64_t ld_x, const void* const w[4], int64_t ld_w, const PackedW& pw,
           const T* bias, const T* lora_a, const T* lora_b, int rank, float lora_scale, T* y,
           int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g, uint8_t* ws, int flags,
           const PeerOut& peers, cudaStream_t stream) {
  if (pair_eligible(M, N_g, rank, y, ld_y, peers, flags) &&
      (!pw.w || (aligned(pw.w, 16) && pw.ld % 2 == 0)))
    return run_pair<T>(dev, x, ld_x, w, ld_w, pw, bias, y, ld_y, M, K_g, N_g, peers, stream);
  if (!w[0]) return QLIN_ERR_ALIGN;  // the other tensor-core paths read planar weights
  if (get_encoder() != QLIN_OK) return QLIN_ERR_LAUNCH;
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const WsLayout L = ws_layout(QLIN_BF16, M, K_g, N_g, rank);
  T* xp = reinterpret_cast<T*>(ws + L.xp_off);
  T* t = rank > 0 ? reinterpret_cast<T*>(ws + L.t_off) : nullptr;
  const int n_tok = n_tok_for(M);
  const bool stack = M <= kStackMaxTokens;
  const int lmode =
      lora_mode(M, rank, K_g, split_for(M, K_g, N_g, rank, dev->num_sms, (flags & QLIN_FLAG_STATIC_WEIGHTS) != 0));
  const bool lora_in = lmode != kLoraPrologue;

  // 1. prologue: component planes of x (plane mode) and the scaled LoRA down
  //    projection; none for stacked mode whose LoRA (if any) runs in the
  //    main kernel
  int after_prologue = 0;
  {
    const int64_t planar_blocks = stack ? 0 : (M * (K_g / 8) + 255) / 256;
    const int rr = stack ? 1 : 8;
    const int64_t lora_blocks = (rank > 0 && !lora_in) ? ((M + 7) / 8) * ((rank + rr - 1) / rr) : 0;
    const int64_t blocks = planar_blocks + lora_blocks;
    if (blocks > INT32_MAX) return QLIN_ERR_SHAPE;
    if (blocks > 0) {
      cudaLaunchConfig_t pc = {};
      pc.gridDim = dim3((unsigned)blocks, 1, 1);
      pc.blockDim = dim3(256, 1, 1);
      pc.stream = stream;
      cudaLaunchAttribute pattr;
      pattr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
      pattr.val.programmaticStreamSerializationAllowed = 1;
      pc.attrs = &pattr;
      pc.numAttrs = 1;
      cudaError_t e = stack ? cudaLaunchKernelEx(&pc, qlin_prologue_kernel<T, 1>, x, ld_x, xp, M, K_g,
                                                 planar_blocks, lora_a, rank, lora_scale, t, L.ld_t)
                            : cudaLaunchKernelEx(&pc, qlin_prologue_kernel<T, 8>, x, ld_x, xp, M, K_g,
                                                 planar_blocks, lora_a, rank, lora_scale, t, L.ld_t);
      if (e != cudaSuccess) return QLIN_ERR_LAUNCH;
      after_prologue = 1;
    }
  }
  // 2. tensor maps
  int sub3d = 0;
  CUtensorMap maps[8];
  std::memset(maps, 0, sizeof(maps));
  for (int p = 0; p < 4; ++p) {
    cuuint64_t dims[2] = {(cuuint64_t)K_g, (cuuint64_t)N_g};
    cuuint64_t strides[1] = {(cuuint64_t)(ld_w * 2)};
    cuuint32_t box[2] = {kTcChunk, kTcBlockO};
    if (encode(&maps[p], dt, 2, const_cast<void*>(w[p]), dims, strides, box) != CUDA_SUCCESS)
      return QLIN_ERR_ALIGN;
  }
  if (!stack) {
    cuuint64_t dims[3] = {(cuuint64_t)K_g, (cuuint64_t)M, 4};
    cuuint64_t strides[2] = {(cuuint64_t)(K_g * 2), (cuuint64_t)(M * K_g * 2)};
    cuuint32_t box[3] = {kTcChunk, (cuuint32_t)n_tok, 1};
    if (encode(&maps[4], dt, 3, xp, dims, strides, box) != CUDA_SUCCESS) return QLIN_ERR_ALIGN;
  } else {
    // raw x rows of a stacked tile: 32 elements (64 bytes, 64-byte swizzle) x n_tok tokens.
    // With K_g a multiple of 8 the four 32-element sub-tiles of a chunk come in
    // one box of a 3-D view [sub-tile (64-byte stride)][token][32 elements]: one
    // TMA operation instead of four (the issue of each TMA operation, not its
    // bytes, set the pace of these small tiles).
    cuuint64_t dims3[3] = {32, (cuuint64_t)M, (cuuint64_t)(K_g / 8)};
    cuuint64_t strides3[2] = {(cuuint64_t)(ld_x * 2), 64};
    cuuint32_t box3[3] = {32, (cuuint32_t)n_tok, 4};
    if (K_g % 8 == 0 && encode(&maps[4], dt, 3, const_cast<T*>(x), dims3, strides3, box3) == CUDA_SUCCESS) {
      sub3d = 1;
    } else {
      cuuint64_t dims[2] = {(cuuint64_t)(4 * K_g), (cuuint64_t)M};
      cuuint64_t strides[1] = {(cuuint64_t)(ld_x * 2)};
      cuuint32_t box[2] = {32, (cuuint32_t)n_tok};
      if (encode(&maps[4], dt, 2, const_cast<T*>(x), dims, strides, box) != CUDA_SUCCESS) return QLIN_ERR_ALIGN;
    }
  }
  int lora_chunks = 0;
  if (rank > 0) {
    cuuint64_t dims[3] = {(cuuint64_t)rank, 4, (cuuint64_t)N_g};
    cuuint64_t strides[2] = {(cuuint64_t)(rank * 2), (cuuint64_t)(4 * rank * 2)};
    cuuint32_t box[3] = {kTcChunk, 1, kTcBlockO};
    if (encode(&maps[5], dt, 3, const_cast<T*>(lora_b), dims, strides, box) != CUDA_SUCCESS)
      return QLIN_ERR_ALIGN;
    cuuint64_t tdims[2] = {(cuuint64_t)rank, (cuuint64_t)M};
    cuuint64_t tstrides[1] = {(cuuint64_t)(L.ld_t * 2)};
    cuuint32_t tbox[2] = {kTcChunk, (cuuint32_t)n_tok};
    if (encode(&maps[6], dt, 2, t, tdims, tstrides, tbox) != CUDA_SUCCESS) return QLIN_ERR_ALIGN;
    lora_chunks = (int)((rank + kTcChunk - 1) / kTcChunk);
    if (lmode == kLoraTc || lmode == kLoraSimt) {
      // lora_a [rank, 4*K_g], rows past rank read as zero: 32-element
      // swizzled columns (tensor-core operand), or plain 256-element row
      // pieces (the CUDA-core mode's slice)
      cuuint64_t adims[2] = {(cuuint64_t)(4 * K_g), (cuuint64_t)rank};
      cuuint64_t astrides[1] = {(cuuint64_t)(4 * K_g * 2)};
      const bool tc = lmode == kLoraTc;
      cuuint32_t abox[2] = {tc ? 32u : (cuuint32_t)kTcLoraSliceBox, (cuuint32_t)kTcLoraInRank};
      // tensor-core mode with the 3-D x view: lora_a's chunk columns likewise in one box
      cuuint64_t adims3[3] = {32, (cuuint64_t)rank, (cuuint64_t)(K_g / 8)};
      cuuint64_t astrides3[2] = {(cuuint64_t)(4 * K_g * 2), 64};
      cuuint32_t abox3[3] = {32, (cuuint32_t)kTcLoraInRank, 4};
      if (tc && sub3d) {
        if (encode(&maps[7], dt, 3, const_cast<T*>(lora_a), adims3, astrides3, abox3) != CUDA_SUCCESS)
          return QLIN_ERR_ALIGN;
      } else if (encode(&maps[7], dt, 2, const_cast<T*>(lora_a), adims, astrides, abox,
                        tc ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE) != CUDA_SUCCESS) {
        return QLIN_ERR_ALIGN;
      }
    }
  }
  // 3. main kernel (+ split-K reduction)
  TcParams prm{};
  prm.x = x;
  prm.ld_x = ld_x;
  prm.bias = bias;
  prm.y = y;
  prm.ld_y = ld_y;
  prm.M = (int)M;
  prm.N_g = (int)N_g;
  prm.K_g = (int)K_g;
  prm.num_chunks = (int)((K_g + kTcChunk - 1) / kTcChunk);
  prm.lora_chunks = lora_chunks;
  prm.split_k = 1;
  prm.partials = nullptr;
  prm.static_weights = (flags & QLIN_FLAG_STATIC_WEIGHTS) ? 1 : 0;
  prm.no_cluster = (flags & QLIN_FLAG_NO_CLUSTER) ? 1 : 0;
  prm.sub3d = sub3d;
  prm.counters = (flags & QLIN_FLAG_ZEROED_WORKSPACE) ? reinterpret_cast<unsigned*>(ws + L.cnt_off)
                                                       : nullptr;
  prm.fuse_reduce = 0;
  prm.after_prologue = after_prologue;
  prm.rank = rank;
  prm.lora_scale = lora_scale;
  prm.lora_a = lora_a;
  prm.ld_a = 4 * K_g;
  prm.peers = peers;
  float4* partials = L.part_bytes ? reinterpret_cast<float4*>(ws + L.part_off) : nullptr;
  switch (n_tok) {
    case 16:
      if (lmode == kLoraSimt) return launch_tc_impl<T, 16, kLoraSimt>(dev, maps, prm, M, K_g, N_g, partials, stream);
      if (lmode == kLoraTc) return launch_tc_impl<T, 16, kLoraTc>(dev, maps, prm, M, K_g, N_g, partials, stream);
      return launch_tc_impl<T, 16, kLoraPrologue>(dev, maps, prm, M, K_g, N_g, partials, stream);
    case 32:
      if (lmode == kLoraTc) return launch_tc_impl<T, 32, kLoraTc>(dev, maps, prm, M, K_g, N_g, partials, stream);
      return launch_tc_impl<T, 32, kLoraPrologue>(dev, maps, prm, M, K_g, N_g, partials, stream);
    case 64: return launch_tc_impl<T, 64, kLoraPrologue>(dev, maps, prm, M, K_g, N_g, partials, stream);
    default: return launch_tc_impl<T, 128, kLoraPrologue>(dev, maps, prm, M, K_g, N_g, partials, stream);
  }
}

template <typename T>
int run_simt(DeviceInfo* dev, const T* x, int64_t ld_x, const void* const w[4], int64_t ld_w,
             const T* bias, const T* lora_a, const T* lora_b, int rank, float lora_scale, T* y,
             int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g, uint8_t* ws, cudaStream_t stream) {
  const WsLayout L = ws_layout(QLIN_F32, M, K_g, N_g, rank);
  float* tf = nullptr;
  if (rank > 0) {
    tf = reinterpret_cast<float*>(ws + L.tf_off);
    dim3 grid((unsigned)((M + 15) / 16), (unsigned)((rank + 7) / 8));
    qlin_lora_down_kernel<T, 16><<<grid, 256, 0, stream>>>(x, ld_x, lora_a, rank, M, 4 * K_g,
                                                            lora_scale, tf, nullptr, 0);
  }
  const T* wr = static_cast<const T*>(w[0]);
  const T* wi = static_cast<const T*>(w[1]);
  const T* wj = static_cast<const T*>(w[2]);
  const T* wk = static_cast<const T*>(w[3]);
  if constexpr (std::is_same<T, float>::value) {
    // fp32 with 16-byte aligned rows: the K-split kernel (float4 loads)
    bool vec = aligned(x, 16) && aligned(y, 16) && ld_x % 4 == 0 && ld_w % 4 == 0 && ld_y % 4 == 0;
    for (int p = 0; p < 4; ++p) vec = vec && aligned(w[p], 16);
    if (vec) {
      // (never above the split the workspace was sized for)
      const int split = std::min(f32_split_for(M, K_g, N_g, dev->num_sms), f32_split_for(M, K_g, N_g, kMaxSms));
      float* part = split > 1 ? reinterpret_cast<float*>(ws + L.part_off) : nullptr;
      if (split > 1 && (!ws || L.part_bytes == 0)) return QLIN_ERR_WORKSPACE;
      dim3 grid((unsigned)((N_g + kSkBO - 1) / kSkBO), (unsigned)((M + kSkBM - 1) / kSkBM), (unsigned)split);
      if (grid.y > 65535) return QLIN_ERR_SHAPE;
      qlin_simt_splitk_kernel<<<grid, 256, 0, stream>>>(x, ld_x, wr, wi, wj, wk, ld_w, bias, tf, lora_b, rank,
                                                        lora_scale, y, ld_y, part, (int)M, (int)K_g, (int)N_g,
                                                        split);
      if (split > 1) {
        const int64_t n = M * N_g;
        qlin_splitk_f32_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
            part, split, bias, tf, lora_b, rank, lora_scale, y, ld_y, (int)M, (int)N_g);
      }
      return QLIN_OK;
    }
  }
  const int64_t big_tiles = ((M + 31) / 32) * ((N_g + 31) / 32);
  if (big_tiles >= dev->num_sms) {
    dim3 grid((unsigned)((N_g + 31) / 32), (unsigned)((M + 31) / 32));
    if (grid.y > 65535) return QLIN_ERR_SHAPE;
    qlin_simt_kernel<T, 32, 32, 16, 2, 2><<<grid, dim3(16, 16), 0, stream>>>(
        x, ld_x, wr, wi, wj, wk, ld_w, bias, tf, lora_b, rank, lora_scale, y, ld_y, M, K_g, N_g);
  } else {
    dim3 grid((unsigned)((N_g + 15) / 16), (unsigned)((M + 15) / 16));
    if (grid.y > 65535) return QLIN_ERR_SHAPE;
    qlin_simt_kernel<T, 16, 16, 16, 1, 1><<<grid, dim3(16, 16), 0, stream>>>(
        x, ld_x, wr, wi, wj, wk, ld_w, bias, tf, lora_b, rank, lora_scale, y, ld_y, M, K_g, N_g);
  }
  return QLIN_OK;
}

template <typename T, int MT, bool LORA, bool PEERS, bool PACKED>
int launch_gemv(DeviceInfo* dev, GemvParams prm, cudaStream_t stream) {
  auto kernel = qlin_gemv_kernel<T, MT, LORA, PEERS, PACKED>;
  const size_t smem = gemv_smem_bytes(MT, prm.nch, LORA);
  const int di = std::is_same<T, __nv_bfloat16>::value ? 0 : 1;
  const int ti = MT == 1 ? 0 : (MT == 2 ? 1 : 2);
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!dev->gemv_attr_set[di][ti][LORA][PEERS][PACKED]) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvMaxSmem) !=
          cudaSuccess)
        return QLIN_ERR_LAUNCH;
      dev->gemv_attr_set[di][ti][LORA][PEERS][PACKED] = true;
    }
  }
  // one output quaternion per row warp, 8 row warps (+ the LoRA warp) per CTA;
  // with LoRA a programmatic dependent of this call's prologue
  const int64_t blocks = (prm.N_g + kGemvWarps - 1) / kGemvWarps;
  if (blocks > INT32_MAX) return QLIN_ERR_SHAPE;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(LORA ? kGemvLoraThreads : kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, prm) == cudaSuccess ? QLIN_OK : QLIN_ERR_LAUNCH;
}

template <typename T, int MT>
int launch_gemv_mt(DeviceInfo* dev, const GemvParams& prm, cudaStream_t stream) {
  if (prm.wq)
    return prm.rank > 0 ? launch_gemv<T, MT, true, false, true>(dev, prm, stream)
                        : launch_gemv<T, MT, false, false, true>(dev, prm, stream);
  return prm.rank > 0 ? launch_gemv<T, MT, true, false, false>(dev, prm, stream)
                      : launch_gemv<T, MT, false, false, false>(dev, prm, stream);
}

// CUDA-core decode kernel: one launch; with LoRA after the down-projection
// prologue, whose t is in the workspace.
template <typename T>
int run_gemv(DeviceInfo* dev, const T* x, int64_t ld_x, const void* const w[4], int64_t ld_w, const PackedW& pw,
             const T* bias, const T* lora_a, const T* lora_b, int rank, float lora_scale, T* y, int64_t ld_y,
             int64_t M, int64_t K_g, int64_t N_g, uint8_t* ws, int flags, const PeerOut& peers,
             cudaStream_t stream) {
  GemvParams prm{};
  prm.x = x;
  prm.ld_x = ld_x;
  for (int p = 0; p < 4; ++p) prm.w[p] = w[p];
  prm.ld_w = ld_w;
  prm.wq = pw.w;
  prm.ld_wq = pw.ld;
  if (!pw.w && !w[0]) return QLIN_ERR_ALIGN;
  prm.bias = bias;
  prm.lora_a = rank > 0 ? lora_a : nullptr;
  prm.lora_b = rank > 0 ? lora_b : nullptr;
  prm.rank = rank;
  prm.lora_scale = lora_scale;
  prm.y = y;
  prm.ld_y = ld_y;
  prm.M = (int)M;
  prm.K_g = (int)K_g;
  prm.N_g = (int)N_g;
  prm.nch = (int)((K_g + kGemvChunk - 1) / kGemvChunk);
  // bulk copies of the x rows need 16-byte aligned rows
  prm.x_bulk = (aligned(x, 16) && (ld_x * 2) % 16 == 0) ? 1 : 0;
  prm.static_weights = (flags & QLIN_FLAG_STATIC_WEIGHTS) ? 1 : 0;
  prm.peers = peers;
  prm.t = nullptr;
  prm.ld_t = 0;
  if (rank > 0) {
    // the scaled LoRA down projection t from the prologue kernel, in the
    // workspace (the same piece the tensor-core path uses)
    if (!ws) return QLIN_ERR_WORKSPACE;
    const WsLayout L = ws_layout(QLIN_BF16, M, K_g, N_g, rank);
    T* t = reinterpret_cast<T*>(ws + L.t_off);
    cudaLaunchAttribute pattr;
    pattr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pattr.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t pc = {};
    pc.gridDim = dim3((unsigned)(((M + 7) / 8) * rank), 1, 1);
    pc.blockDim = dim3(256, 1, 1);
    pc.stream = stream;
    pc.attrs = &pattr;
    pc.numAttrs = 1;
    if (cudaLaunchKernelEx(&pc, qlin_prologue_kernel<T, 1>, x, ld_x, static_cast<T*>(nullptr), M, K_g,
                           (int64_t)0, lora_a, rank, lora_scale, t, L.ld_t) != cudaSuccess)
      return QLIN_ERR_LAUNCH;
    prm.t = t;
    prm.ld_t = L.ld_t;
  }
  switch (gemv_tokens(M)) {
    case 1: return launch_gemv_mt<T, 1>(dev, prm, stream);
    case 2: return launch_gemv_mt<T, 2>(dev, prm, stream);
    default: return launch_gemv_mt<T, 4>(dev, prm, stream);
  }
}

template <typename T>
int dispatch(int algo, DeviceInfo* dev, const void* x, int64_t ld_x, const void* const w[4],
             int64_t ld_w, const PackedW& pw, const void* bias, const void* lora_a, const void* lora_b, int rank,
             float lora_scale, void* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g,
             uint8_t* ws, int flags, const PeerOut& peers, cudaStream_t stream) {
  const T* xt = static_cast<const T*>(x);
  const T* bt = static_cast<const T*>(bias);
  const T* la = static_cast<const T*>(lora_a);
  const T* lb = static_cast<const T*>(lora_b);
  T* yt = static_cast<T*>(y);
  // peer outputs (column-partitioned layer) are written by the tensor-core path only
  if (!w[0] && (algo == QLIN_ALGO_SIMT || std::is_same<T, float>::value)) return QLIN_ERR_ALIGN;
  if constexpr (std::is_same<T, float>::value) {
    if (has_peers(peers)) return QLIN_ERR_ALIGN;
    return run_simt<T>(dev, xt, ld_x, w, ld_w, bt, la, lb, rank, lora_scale, yt, ld_y, M, K_g, N_g, ws,
                       stream);
  } else {
    // peer outputs (the fused all-gather) are written by the tensor-core kernel only
    if (algo == QLIN_ALGO_GEMV && has_peers(peers)) return QLIN_ERR_ALIGN;
    if (algo == QLIN_ALGO_GEMV)
      return run_gemv<T>(dev, xt, ld_x, w, ld_w, pw, bt, la, lb, rank, lora_scale, yt, ld_y, M, K_g, N_g, ws, flags,
                         peers, stream);
    if (algo == QLIN_ALGO_TC)
      return run_tc<T>(dev, xt, ld_x, w, ld_w, pw, bt, la, lb, rank, lora_scale, yt, ld_y, M, K_g, N_g, ws,
                       flags, peers, stream);
    if (has_peers(peers)) return QLIN_ERR_ALIGN;
    return run_simt<T>(dev, xt, ld_x, w, ld_w, bt, la, lb, rank, lora_scale, yt, ld_y, M, K_g, N_g, ws,
                       stream);
  }
}

template <typename T, int N_TOK>
int plan_tc(DeviceInfo* dev, int64_t M, int64_t K_g, int64_t N_g, int rank, int flags, int* split,
            int* resident) {
  *split = split_for(M, K_g, N_g, rank, dev->num_sms, (flags & QLIN_FLAG_STATIC_WEIGHTS) != 0);
  const int li = lora_mode(M, rank, K_g, *split);
  int st = QLIN_OK;
  if constexpr (N_TOK == 16) {
    st = li == kLoraSimt ? ensure_tc_attrs<T, N_TOK, kLoraSimt>(dev)
                         : (li == kLoraTc ? ensure_tc_attrs<T, N_TOK, kLoraTc>(dev)
                                          : ensure_tc_attrs<T, N_TOK, kLoraPrologue>(dev));
  } else if constexpr (N_TOK == 32) {
    st = li == kLoraTc ? ensure_tc_attrs<T, N_TOK, kLoraTc>(dev) : ensure_tc_attrs<T, N_TOK, kLoraPrologue>(dev);
  } else {
    st = ensure_tc_attrs<T, N_TOK, kLoraPrologue>(dev);
  }
  if (st != QLIN_OK) return st;
  const int ti = n_tok_index(N_TOK);
  const int di = std::is_same<T, __nv_bfloat16>::value ? 0 : 1;
  *resident = dev->resident[di][ti][li][0][0];
  return QLIN_OK;
}

// qlin_forward_ex, with every output also stored to the peers' outputs.
static int forward_common(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi,
                          const void* wj, const void* wk, int64_t ld_w, const void* bias, const void* lora_a,
                          const void* lora_b, int rank, float lora_scale, void* y, int64_t ld_y, int64_t M,
                          int64_t K_g, int64_t N_g, void* workspace, size_t workspace_bytes, int algo, int flags,
                          void* stream, const PeerOut& peers, const PackedW& packed = PackedW()) {
  int st = validate(dtype, x, ld_x, wr, wi, wj, wk, ld_w, lora_a, lora_b, rank, y, ld_y, M, K_g, N_g, &packed);
  if (st != QLIN_OK) return st;
  if (M == 0) return QLIN_OK;
  if (algo < QLIN_ALGO_AUTO || algo > QLIN_ALGO_GEMV) return QLIN_ERR_ARG;
  if (flags & ~(QLIN_FLAG_STATIC_WEIGHTS | QLIN_FLAG_ZEROED_WORKSPACE | QLIN_FLAG_NO_PAIR |
                QLIN_FLAG_NO_CLUSTER)) return QLIN_ERR_ARG;
  if (rank == 0) lora_a = lora_b = nullptr;
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st != QLIN_OK) return st;
  const void* w[4] = {wr, wi, wj, wk};
  // The packed weight cache serves the kernels that read it (the decode GEMV
  // and the CTA-pair kernel): 16-bit types, a 16-byte aligned buffer, an even
  // row length; the other paths read the planar weights.
  PackedW pw = packed;
  if (pw.w && (dtype == QLIN_F32 || !aligned(pw.w, 16) || pw.ld % 2 != 0 || K_g % 8 != 0)) pw = PackedW();
  if (!pw.w && !wr) return QLIN_ERR_ALIGN;
  // the packed GEMV does not read the planar weights: their alignment does not count
  const void* const wnone[4] = {nullptr, nullptr, nullptr, nullptr};
  const void* const* wg = pw.w ? wnone : w;
  if (algo == QLIN_ALGO_AUTO) {
    algo = select_algo(dtype);
    if (algo == QLIN_ALGO_TC && gemv_auto(M, N_g, rank, dev) &&
        gemv_eligible(dtype, x, ld_x, wg, ld_w, bias, lora_a, lora_b, rank, y, ld_y, M, K_g))
      algo = QLIN_ALGO_GEMV;
    else if (algo == QLIN_ALGO_TC &&
             !tc_eligible(dtype, x, ld_x, w, ld_w, lora_a, lora_b, rank, y, ld_y, K_g))
      algo = QLIN_ALGO_SIMT;
  } else if (algo == QLIN_ALGO_TC &&
             !tc_eligible(dtype, x, ld_x, w, ld_w, lora_a, lora_b, rank, y, ld_y, K_g)) {
    return QLIN_ERR_ALIGN;
  } else if (algo == QLIN_ALGO_GEMV &&
             !gemv_eligible(dtype, x, ld_x, wg, ld_w, bias, lora_a, lora_b, rank, y, ld_y, M, K_g)) {
    return QLIN_ERR_ALIGN;
  }
  const WsLayout L = ws_layout(dtype, M, K_g, N_g, rank);
  if (L.total > 0 && (!workspace || workspace_bytes < L.total || !aligned(workspace, 256)))
    return QLIN_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaGetLastError();  // clear stale errors so the check below is this call's
  switch (dtype) {
    case QLIN_F32:
      st = dispatch<float>(algo, dev, x, ld_x, w, ld_w, pw, bias, lora_a, lora_b, rank, lora_scale, y, ld_y, M,
                           K_g, N_g, ws, flags, peers, s);
      break;
    case QLIN_BF16:
      st = dispatch<__nv_bfloat16>(algo, dev, x, ld_x, w, ld_w, pw, bias, lora_a, lora_b, rank, lora_scale, y,
                                   ld_y, M, K_g, N_g, ws, flags, peers, s);
      break;
    default:
      st = dispatch<__half>(algo, dev, x, ld_x, w, ld_w, pw, bias, lora_a, lora_b, rank, lora_scale, y, ld_y, M,
                            K_g, N_g, ws, flags, peers, s);
      break;
  }
  if (st != QLIN_OK) return st;
  return cudaGetLastError() == cudaSuccess ? QLIN_OK : QLIN_ERR_LAUNCH;
}

// NCCL, resolved at run time: the library the process already loaded (a
// host framework's, so that one NCCL serves the whole process), else
// libnccl.so.2.  Only qlin_sharded_fwd and the bootstrap helpers use it; the
// rest of the library loads and runs without NCCL.
struct NcclApi {
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  bool tried = false;
};
NcclApi g_nccl;

const NcclApi* nccl_api() {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_nccl.tried) {
    g_nccl.tried = true;
    // RTLD_DEFAULT is a null handle: resolve through it when it sees NCCL
    auto resolve = [](void* h) {
      g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(dlsym(h, "ncclAllGather"));
      g_nccl.unique_id = reinterpret_cast<decltype(g_nccl.unique_id)>(dlsym(h, "ncclGetUniqueId"));
      g_nccl.comm_init = reinterpret_cast<decltype(g_nccl.comm_init)>(dlsym(h, "ncclCommInitRank"));
      g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
      return g_nccl.all_gather && g_nccl.unique_id && g_nccl.comm_init && g_nccl.comm_destroy;
    };
    if (!resolve(RTLD_DEFAULT)) {
      void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
      if (h) resolve(h);
    }
  }
  return (g_nccl.all_gather && g_nccl.unique_id && g_nccl.comm_init && g_nccl.comm_destroy) ? &g_nccl : nullptr;
}

// Device staging of qlin_forward_host: x [M][4 K_g] and y [M][4 N_g], each
// 256-byte aligned, ahead of the forward's own workspace.
size_t host_staging_bytes(int dtype, int64_t M, int64_t K_g, int64_t N_g) {
  const int64_t es = (int64_t)elem_size(dtype);
  return (size_t)(round_up(M * 4 * K_g * es, 256) + round_up(M * 4 * N_g * es, 256));
}

// Largest transfer qlin_forward_host runs without the copy engine (the x
// stage-in kernel, y stored by the kernels through the host mapping).
constexpr size_t kHostDirectBytes = 64 * 1024;

// The device address of a page-locked host buffer when qlin_forward_host may
// move it with a kernel: mapped into the device's address space, at most
// kHostDirectBytes of rows, rows and leading dimension in whole 16-byte
// words, 16-byte aligned; else null (a copy-engine transfer).
void* direct_host_map(const void* p, size_t row_bytes, size_t ld_bytes, int64_t M) {
  if (row_bytes * (size_t)M > kHostDirectBytes || row_bytes % 16 || ld_bytes % 16 || !aligned(p, 16)) return nullptr;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// A small kernel as a programmatic dependent of the previous kernel of the stream.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned blocks, cudaStream_t s, Args... args) {
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Workspace of qlin_sharded_fwd: the gathered column blocks [world][M][4 N_g]
// (M > 1), then the single-GPU forward's workspace.
size_t sharded_gather_bytes(int dtype, int64_t M, int64_t N_g, int world) {
  return M > 1 ? (size_t)round_up((int64_t)world * M * 4 * N_g * elem_size(dtype), 256) : 0;
}

// One rank's shard of the column-partitioned layer with its outputs stored
// into every rank's full output (peer stores or one multicast store each),
// between an entry and an exit flag barrier over the ranks' flag arrays.
int allgather_common(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi, const void* wj,
                     const void* wk, int64_t ld_w, const void* bias, const void* lora_a, const void* lora_b, int rank,
                     float lora_scale, int64_t M, int64_t K_g, int64_t N_g, void* workspace, size_t workspace_bytes,
                     int flags, int world, int world_rank, void* y, int64_t ld_out, const PeerOut& peers,
                     unsigned* const* flag_arrays, unsigned* epoch_word, void* stream) {
  if (world > 1 && (!flag_arrays || !epoch_word)) return QLIN_ERR_ARG;
  for (int q = 0; q < world; ++q)
    if (world > 1 && !flag_arrays[q]) return QLIN_ERR_ARG;
  int st = validate(dtype, x, ld_x, wr, wi, wj, wk, ld_w, lora_a, lora_b, rank, y, ld_out, M, K_g, N_g);
  if (st != QLIN_OK || M == 0) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PeerFlags pf;
  for (int q = 0; q < world; ++q) pf.f[q] = world > 1 ? flag_arrays[q] : nullptr;
  if (world > 1) {
    // Entry barrier (slots [world, 2*world), epoch word 1): no rank stores
    // into a peer's output while that peer's work queued after the previous
    // call (reading that output) may still be running.
    cudaGetLastError();
    qlin_peer_barrier_kernel<<<1, 32, 0, s>>>(pf, epoch_word + 1, world_rank, world, world);
    if (cudaGetLastError() != cudaSuccess) return QLIN_ERR_LAUNCH;
  }
  st = forward_common(dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale, y, ld_out, M,
                      K_g, N_g, workspace, workspace_bytes, QLIN_ALGO_TC, flags, stream, peers);
  if (st != QLIN_OK || world == 1) return st;
  // Exit barrier (slots [0, world), epoch word 0): every rank's columns are
  // in every rank's output.
  qlin_peer_barrier_kernel<<<1, 32, 0, s>>>(pf, epoch_word, world_rank, world, 0);
  return cudaGetLastError() == cudaSuccess ? QLIN_OK : QLIN_ERR_LAUNCH;
}

}  // namespace

extern "C" {

const char* qlin_status_string(int status) {
  switch (status) {
    case QLIN_OK: return "ok";
    case QLIN_ERR_SHAPE: return "invalid shape or leading dimension";
    case QLIN_ERR_DTYPE: return "unsupported dtype";
    case QLIN_ERR_ALIGN: return "pointer or leading-dimension alignment not supported by this path";
    case QLIN_ERR_WORKSPACE: return "workspace missing or too small";
    case QLIN_ERR_LAUNCH: return "CUDA launch or runtime error";
    case QLIN_ERR_DEVICE: return "current device is not sm_100 (B200 class)";
    case QLIN_ERR_TIMEOUT: return "a bounded device-side wait ran out";
    case QLIN_ERR_ARG: return "null pointer or invalid option";
    case QLIN_ERR_COLLECTIVE: return "NCCL not loadable, or an NCCL call failed";
    default: return "unknown status";
  }
}

int qlin_abi_version(void) { return 104; }

int qlin_workspace_size(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank, size_t* bytes) {
  if (!bytes) return QLIN_ERR_ARG;
  if (dtype != QLIN_F32 && dtype != QLIN_BF16 && dtype != QLIN_F16) return QLIN_ERR_DTYPE;
  if (M < 0 || K_g <= 0 || N_g <= 0 || rank < 0) return QLIN_ERR_SHAPE;
  *bytes = ws_layout(dtype, M, K_g, N_g, rank).total;
  return QLIN_OK;
}

int qlin_select_algo(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank) {
  (void)M; (void)K_g; (void)N_g; (void)rank;
  return select_algo(dtype);
}

int qlin_plan(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank, int flags, int* algo,
              int* tile_tokens, int* split_k, int* launches, int* resident_ctas) {
  if (dtype != QLIN_F32 && dtype != QLIN_BF16 && dtype != QLIN_F16) return QLIN_ERR_DTYPE;
  if (flags & ~(QLIN_FLAG_STATIC_WEIGHTS | QLIN_FLAG_ZEROED_WORKSPACE | QLIN_FLAG_NO_PAIR |
                QLIN_FLAG_NO_CLUSTER)) return QLIN_ERR_ARG;
  if (M <= 0 || K_g <= 0 || N_g <= 0 || rank < 0) return QLIN_ERR_SHAPE;
  DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != QLIN_OK) return st;
  int a = (dtype == QLIN_F32 || K_g % 8 != 0 || (rank > 0 && rank % 8 != 0)) ? QLIN_ALGO_SIMT
                                                                               : QLIN_ALGO_TC;
  if (a == QLIN_ALGO_TC && gemv_auto(M, N_g, rank, dev) && rank <= kGemvMaxRank && rank % 4 == 0 &&
      gemv_smem_bytes(gemv_tokens(M), (int)((K_g + kGemvChunk - 1) / kGemvChunk), rank > 0) <= kGemvMaxSmem)
    a = QLIN_ALGO_GEMV;
  int nt = 0, sp = 1, res = 0, nl = 0;
  if (a == QLIN_ALGO_GEMV) {
    nt = gemv_tokens(M);
    nl = rank > 0 ? 2 : 1;  // LoRA: the down-projection prologue, then the decode kernel
    int per_sm = 0;
    const size_t smem = gemv_smem_bytes(nt, (int)((K_g + kGemvChunk - 1) / kGemvChunk), rank > 0);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qlin_gemv_kernel<__nv_bfloat16, 1, false, false>,
                                                      kGemvThreads, smem) != cudaSuccess)
      per_sm = 0;
    cudaGetLastError();
    res = per_sm * dev->num_sms;
  } else if (a == QLIN_ALGO_TC && M > kStackMaxTokens && rank == 0 && N_g % 2 == 0 &&
             !(flags & QLIN_FLAG_NO_PAIR)) {
    // the CTA-pair kernel (assuming a 16-byte aligned output)
    int cap = 0;
    const bool big = pair_tokens(M) == 256;
    st = dtype == QLIN_BF16 ? (big ? pair_attrs<__nv_bfloat16, false, 256>(dev, &cap)
                                   : pair_attrs<__nv_bfloat16, false, 128>(dev, &cap))
                            : (big ? pair_attrs<__half, false, 256>(dev, &cap) : pair_attrs<__half, false, 128>(dev, &cap));
    if (st != QLIN_OK) return st;
    a = QLIN_PLAN_TC_PAIR;
    nt = pair_tokens(M);
    nl = 1;
    res = 2 * (int)std::min<int64_t>(pair_tiles(M, N_g), cap);
  } else if (a == QLIN_ALGO_TC) {
    nt = n_tok_for(M);
    const bool bf = dtype == QLIN_BF16;
    switch (nt) {
      case 16: st = bf ? plan_tc<__nv_bfloat16, 16>(dev, M, K_g, N_g, rank, flags, &sp, &res)
                       : plan_tc<__half, 16>(dev, M, K_g, N_g, rank, flags, &sp, &res); break;
      case 32: st = bf ? plan_tc<__nv_bfloat16, 32>(dev, M, K_g, N_g, rank, flags, &sp, &res)
                       : plan_tc<__half, 32>(dev, M, K_g, N_g, rank, flags, &sp, &res); break;
      case 64: st = bf ? plan_tc<__nv_bfloat16, 64>(dev, M, K_g, N_g, rank, flags, &sp, &res)
                       : plan_tc<__half, 64>(dev, M, K_g, N_g, rank, flags, &sp, &res); break;
      default: st = bf ? plan_tc<__nv_bfloat16, 128>(dev, M, K_g, N_g, rank, flags, &sp, &res)
                       : plan_tc<__half, 128>(dev, M, K_g, N_g, rank, flags, &sp, &res); break;
    }
    if (st != QLIN_OK) return st;
    bool clustered = false;
    if (nt == 16 && !(flags & QLIN_FLAG_NO_CLUSTER)) {
      const int lm = lora_mode(M, rank, K_g, sp);
      const int64_t tiles = (N_g + kTcBlockO - 1) / kTcBlockO;
      int cs = 0;
      if (lm == kLoraSimt)
        cs = bf ? cluster_split<__nv_bfloat16, kLoraSimt>(dev, M, K_g, sp, tiles)
                : cluster_split<__half, kLoraSimt>(dev, M, K_g, sp, tiles);
      else if (lm == kLoraTc)
        cs = bf ? cluster_split<__nv_bfloat16, kLoraTc>(dev, M, K_g, sp, tiles)
                : cluster_split<__half, kLoraTc>(dev, M, K_g, sp, tiles);
      else
        cs = bf ? cluster_split<__nv_bfloat16, kLoraPrologue>(dev, M, K_g, sp, tiles)
                : cluster_split<__half, kLoraPrologue>(dev, M, K_g, sp, tiles);
      if (cs > 0) {
        clustered = true;
        sp = cs;
      }
    }
    const bool fused = clustered || ((flags & QLIN_FLAG_ZEROED_WORKSPACE) && M <= kFusedReduceMaxTokens);
    const bool prologue = M > kStackMaxTokens || (rank > 0 && lora_mode(M, rank, K_g, sp) == kLoraPrologue);
    nl = 1 + (prologue ? 1 : 0) + ((sp > 1 && !fused) ? 1 : 0);
  } else {
    // CUDA-core kernel (+ the LoRA down projection; fp32: + the K-split reduction)
    nl = rank > 0 ? 2 : 1;
    if (dtype == QLIN_F32) {
      sp = std::min(f32_split_for(M, K_g, N_g, dev->num_sms), f32_split_for(M, K_g, N_g, kMaxSms));
      nt = kSkBM;
      if (sp > 1) nl += 1;
    }
  }
  if (algo) *algo = a;
  if (tile_tokens) *tile_tokens = nt;
  if (split_k) *split_k = sp;
  if (launches) *launches = nl;
  if (resident_ctas) *resident_ctas = res;
  return QLIN_OK;
}

int qlin_forward_ex(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi, const void* wj,
                    const void* wk, int64_t ld_w, const void* bias, const void* lora_a, const void* lora_b,
                    int rank, float lora_scale, void* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g,
                    void* workspace, size_t workspace_bytes, int algo, int flags, void* stream) {
  PeerOut none;
  none.n = 0;
  return forward_common(dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale, y, ld_y,
                        M, K_g, N_g, workspace, workspace_bytes, algo, flags, stream, none);
}

int qlin_forward_packed(int dtype, const void* x, int64_t ld_x, const void* wq, int64_t ld_wq, const void* wr,
                        const void* wi, const void* wj, const void* wk, int64_t ld_w, const void* bias,
                        const void* lora_a, const void* lora_b, int rank, float lora_scale, void* y, int64_t ld_y,
                        int64_t M, int64_t K_g, int64_t N_g, void* workspace, size_t workspace_bytes, int flags,
                        void* stream) {
  if (!wq && M > 0) return QLIN_ERR_ARG;
  PeerOut none;
  none.n = 0;
  PackedW pw;
  pw.w = wq;
  pw.ld = ld_wq;
  return forward_common(dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale, y, ld_y,
                        M, K_g, N_g, workspace, workspace_bytes, QLIN_ALGO_AUTO, flags, stream, none, pw);
}

int qlin_forward_allgather(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi,
                           const void* wj, const void* wk, int64_t ld_w, const void* bias, const void* lora_a,
                           const void* lora_b, int rank, float lora_scale, int64_t M, int64_t K_g, int64_t N_g,
                           void* workspace, size_t workspace_bytes, int flags, int world, int world_rank,
                           void* const* outs, int64_t ld_out, int64_t col_offset, unsigned* const* flag_arrays,
                           unsigned* epoch_word, void* stream) {
  if (dtype != QLIN_BF16 && dtype != QLIN_F16) return QLIN_ERR_DTYPE;
  if (world < 1 || world > kMaxPeers + 1 || world_rank < 0 || world_rank >= world) return QLIN_ERR_ARG;
  if (!outs) return QLIN_ERR_ARG;
  for (int q = 0; q < world; ++q)
    if (!outs[q]) return QLIN_ERR_ARG;
  if (col_offset < 0 || col_offset % 4 != 0 || ld_out < col_offset + 4 * N_g) return QLIN_ERR_SHAPE;
  PeerOut peers;
  for (int q = 0; q < world; ++q)
    if (q != world_rank) peers.y[peers.n++] = static_cast<uint8_t*>(outs[q]) + col_offset * 2;
  void* y = static_cast<uint8_t*>(outs[world_rank]) + col_offset * 2;
  return allgather_common(dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale, M, K_g, N_g,
                          workspace, workspace_bytes, flags, world, world_rank, y, ld_out, peers, flag_arrays,
                          epoch_word, stream);
}

int qlin_forward_allgather_mc(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi,
                              const void* wj, const void* wk, int64_t ld_w, const void* bias, const void* lora_a,
                              const void* lora_b, int rank, float lora_scale, int64_t M, int64_t K_g, int64_t N_g,
                              void* workspace, size_t workspace_bytes, int flags, int world, int world_rank,
                              void* out, void* out_mc, int64_t ld_out, int64_t col_offset,
                              unsigned* const* flag_arrays, unsigned* epoch_word, void* stream) {
  if (dtype != QLIN_BF16 && dtype != QLIN_F16) return QLIN_ERR_DTYPE;
  if (world < 1 || world > kMaxPeers + 1 || world_rank < 0 || world_rank >= world) return QLIN_ERR_ARG;
  if (!out || !out_mc) return QLIN_ERR_ARG;
  if (col_offset < 0 || col_offset % 4 != 0 || ld_out < col_offset + 4 * N_g) return QLIN_ERR_SHAPE;
  PeerOut peers;
  peers.mc = static_cast<uint8_t*>(out_mc) + col_offset * 2;
  void* y = static_cast<uint8_t*>(out) + col_offset * 2;
  return allgather_common(dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale, M, K_g, N_g,
                          workspace, workspace_bytes, flags, world, world_rank, y, ld_out, peers, flag_arrays,
                          epoch_word, stream);
}

int qlin_ipc_alloc(size_t bytes, void** out, void* handle) {
  if (!out || !handle || bytes == 0) return QLIN_ERR_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return QLIN_ERR_LAUNCH;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return QLIN_ERR_LAUNCH;
  }
  std::memcpy(handle, &h, sizeof(h));
  *out = p;
  return QLIN_OK;
}

int qlin_ipc_free(void* p) {
  if (!p) return QLIN_ERR_ARG;
  return cudaFree(p) == cudaSuccess ? QLIN_OK : QLIN_ERR_LAUNCH;
}

int qlin_ipc_open(const void* handle, int64_t offset, void** out) {
  if (!handle || !out || offset < 0) return QLIN_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess || !base)
    return QLIN_ERR_LAUNCH;
  *out = static_cast<uint8_t*>(base) + offset;
  return QLIN_OK;
}

int qlin_ipc_close(void* base) {
  if (!base) return QLIN_ERR_ARG;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? QLIN_OK : QLIN_ERR_LAUNCH;
}

int qlin_forward(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi, const void* wj,
                 const void* wk, int64_t ld_w, const void* bias, const void* lora_a, const void* lora_b,
                 int rank, float lora_scale, void* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g,
                 void* workspace, size_t workspace_bytes, void* stream) {
  return qlin_forward_ex(dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale, y,
                         ld_y, M, K_g, N_g, workspace, workspace_bytes, QLIN_ALGO_AUTO, 0, stream);
}

int qlin_get_device_error(void* stream, int clear, int* device_status) {
  if (!device_status) return QLIN_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return QLIN_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, qlin::g_device_error, sizeof(int)) != cudaSuccess) return QLIN_ERR_LAUNCH;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(qlin::g_device_error, &zero, sizeof(int)) != cudaSuccess) return QLIN_ERR_LAUNCH;
  }
  *device_status = v;
  return QLIN_OK;
}

int qlin_gather_columns(int dtype, const void* src, void* dst, int64_t G, int64_t M, int64_t n_shard,
                        int64_t ld_dst, void* stream) {
  if (dtype != QLIN_F32 && dtype != QLIN_BF16 && dtype != QLIN_F16) return QLIN_ERR_DTYPE;
  if (G <= 0 || M < 0 || n_shard <= 0 || ld_dst < G * n_shard) return QLIN_ERR_SHAPE;
  if (M == 0) return QLIN_OK;
  if (!src || !dst) return QLIN_ERR_ARG;
  DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != QLIN_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t total = G * M * n_shard;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)dev->num_sms * 16);
  cudaGetLastError();
  if (elem_size(dtype) == 4)
    qlin_gather_kernel<uint32_t><<<blocks, 256, 0, s>>>(static_cast<const uint32_t*>(src),
                                                        static_cast<uint32_t*>(dst), G, M, n_shard, ld_dst);
  else
    qlin_gather_kernel<uint16_t><<<blocks, 256, 0, s>>>(static_cast<const uint16_t*>(src),
                                                        static_cast<uint16_t*>(dst), G, M, n_shard, ld_dst);
  return cudaGetLastError() == cudaSuccess ? QLIN_OK : QLIN_ERR_LAUNCH;
}

int qlin_host_workspace_size(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank, size_t* bytes) {
  if (!bytes) return QLIN_ERR_ARG;
  size_t local = 0;
  const int st = qlin_workspace_size(dtype, M, K_g, N_g, rank, &local);
  if (st != QLIN_OK) return st;
  *bytes = host_staging_bytes(dtype, M, K_g, N_g) + local;
  return QLIN_OK;
}

int qlin_forward_host(int dtype, const void* x_host, int64_t ld_x, const void* wr, const void* wi, const void* wj,
                      const void* wk, int64_t ld_w, const void* bias, const void* lora_a, const void* lora_b,
                      int rank, float lora_scale, void* y_host, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g,
                      void* workspace, size_t workspace_bytes, int algo, int flags, void* stream) {
  if (dtype != QLIN_F32 && dtype != QLIN_BF16 && dtype != QLIN_F16) return QLIN_ERR_DTYPE;
  if (M < 0 || K_g <= 0 || N_g <= 0 || ld_x < 4 * K_g || ld_y < 4 * N_g) return QLIN_ERR_SHAPE;
  if (M == 0) return QLIN_OK;
  if (!x_host || !y_host) return QLIN_ERR_ARG;
  const size_t es = elem_size(dtype), staging = host_staging_bytes(dtype, M, K_g, N_g);
  if (!workspace || workspace_bytes < staging) return QLIN_ERR_WORKSPACE;
  uint8_t* xd = static_cast<uint8_t*>(workspace);
  uint8_t* yd = xd + round_up(M * 4 * K_g * (int64_t)es, 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t xrow = (size_t)(4 * K_g) * es, yrow = (size_t)(4 * N_g) * es;
  // Decode-sized transfers between page-locked, device-mapped host buffers
  // and the device: x by a small kernel of the dependent-launch chain, y
  // stored by the layer's own kernels; larger or pageable ones as
  // copy-engine transfers.
  void* xmap = direct_host_map(x_host, xrow, (size_t)ld_x * es, M);
  void* ymap = direct_host_map(y_host, yrow, (size_t)ld_y * es, M);
  cudaError_t e;
  if (xmap) {
    const int64_t row = (int64_t)(xrow / 16), n = M * row;
    e = launch_pdl(qlin_stage_in_kernel, (unsigned)((n + 511) / 512), s, static_cast<const uint4*>(xmap),
                   (int64_t)(ld_x * es / 16), reinterpret_cast<uint4*>(xd), row, row, M);
  } else {
    // one copy when the host rows are contiguous, else a strided one
    e = ld_x == 4 * K_g
            ? cudaMemcpyAsync(xd, x_host, xrow * M, cudaMemcpyHostToDevice, s)
            : cudaMemcpy2DAsync(xd, xrow, x_host, (size_t)ld_x * es, xrow, (size_t)M, cudaMemcpyHostToDevice, s);
  }
  if (e != cudaSuccess) return QLIN_ERR_LAUNCH;
  // a decode-sized output goes straight from the kernels' epilogues into the
  // page-locked host buffer through its device mapping
  const int st = qlin_forward_ex(dtype, xd, 4 * K_g, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale,
                                 ymap ? ymap : yd, ymap ? ld_y : 4 * N_g, M, K_g, N_g, xd + staging,
                                 workspace_bytes - staging, algo, flags, stream);
  if (st != QLIN_OK) return st;
  if (ymap) {
    e = cudaSuccess;
  } else {
    e = ld_y == 4 * N_g
            ? cudaMemcpyAsync(y_host, yd, yrow * M, cudaMemcpyDeviceToHost, s)
            : cudaMemcpy2DAsync(y_host, (size_t)ld_y * es, yd, yrow, yrow, (size_t)M, cudaMemcpyDeviceToHost, s);
  }
  return e == cudaSuccess ? QLIN_OK : QLIN_ERR_LAUNCH;
}

int qlin_sharded_workspace_size(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank, int world,
                                size_t* bytes) {
  if (!bytes || world < 1) return QLIN_ERR_ARG;
  size_t local = 0;
  const int st = qlin_workspace_size(dtype, M, K_g, N_g, rank, &local);
  if (st != QLIN_OK) return st;
  *bytes = sharded_gather_bytes(dtype, M, N_g, world) + local;
  return QLIN_OK;
}

int qlin_sharded_fwd(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi, const void* wj,
                     const void* wk, int64_t ld_w, const void* bias, const void* lora_a, const void* lora_b,
                     int rank, float lora_scale, void* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g,
                     void* workspace, size_t workspace_bytes, int flags, void* nccl_comm, int world,
                     int world_rank, void* stream) {
  if (world < 1 || world_rank < 0 || world_rank >= world || !nccl_comm) return QLIN_ERR_ARG;
  if (dtype != QLIN_F32 && dtype != QLIN_BF16 && dtype != QLIN_F16) return QLIN_ERR_DTYPE;
  if (M < 0 || N_g <= 0 || ld_y < (int64_t)world * 4 * N_g) return QLIN_ERR_SHAPE;
  const int64_t cols = 4 * N_g;  // this rank's output columns
  const size_t es = elem_size(dtype);
  // this rank's columns: for one token straight into its place in y (the
  // all-gather then runs in place), else into its block of the gathered buffer
  const size_t gather = sharded_gather_bytes(dtype, M, N_g, world);
  if (M > 1 && (!workspace || workspace_bytes < gather)) return QLIN_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* blocks = M > 1 ? ws : static_cast<uint8_t*>(y);
  uint8_t* mine = blocks + (size_t)world_rank * (M > 1 ? M * cols : cols) * es;
  int st = qlin_forward_ex(dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale, mine,
                           M > 1 ? cols : ld_y, M, K_g, N_g, ws ? ws + gather : nullptr,
                           workspace_bytes > gather ? workspace_bytes - gather : 0, QLIN_ALGO_AUTO, flags, stream);
  if (st != QLIN_OK || M == 0) return st;
  const NcclApi* nc = nccl_api();
  if (!nc) return QLIN_ERR_COLLECTIVE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // in place: rank r's block is already at offset r * count of the receive buffer
  if (nc->all_gather(mine, blocks, (size_t)(M > 1 ? M * cols : cols) * es, ncclUint8,
                     static_cast<ncclComm_t>(nccl_comm), s) != ncclSuccess)
    return QLIN_ERR_COLLECTIVE;
  if (M == 1) return QLIN_OK;
  return qlin_gather_columns(dtype, blocks, y, world, M, cols, ld_y, stream);
}

int qlin_nccl_unique_id(void* id) {
  if (!id) return QLIN_ERR_ARG;
  const NcclApi* nc = nccl_api();
  if (!nc) return QLIN_ERR_COLLECTIVE;
  ncclUniqueId u;
  if (nc->unique_id(&u) != ncclSuccess) return QLIN_ERR_COLLECTIVE;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(id, &u, sizeof(u));
  return QLIN_OK;
}

int qlin_nccl_comm_init(void** comm, int world, const void* id, int world_rank) {
  if (!comm || !id || world < 1 || world_rank < 0 || world_rank >= world) return QLIN_ERR_ARG;
  const NcclApi* nc = nccl_api();
  if (!nc) return QLIN_ERR_COLLECTIVE;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  if (nc->comm_init(&c, world, u, world_rank) != ncclSuccess) return QLIN_ERR_COLLECTIVE;
  *comm = c;
  return QLIN_OK;
}

int qlin_nccl_comm_destroy(void* comm) {
  if (!comm) return QLIN_ERR_ARG;
  const NcclApi* nc = nccl_api();
  if (!nc) return QLIN_ERR_COLLECTIVE;
  return nc->comm_destroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? QLIN_OK : QLIN_ERR_COLLECTIVE;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory at the point where they run
// the layer: code that must not call cudaMalloc mid-stream (it can
// synchronise the device), plugins of host frameworks that hand out only
// input and output buffers, and runtimes that forbid allocation after
// start-up.  qlin_forward_noalloc serves them with the same kernels as
// qlin_forward, taking its scratch from a fixed buffer compiled into this
// library instead of a caller-provided workspace.
// ---------------------------------------------------------------------------

// The fixed scratch buffer.  Every GPU that loads this library holds it until
// the process exits; every call on a device shares it.  In host code the name
// is only a stand-in: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[QLIN_NOALLOC_SCRATCH_BYTES];

namespace {

void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch for the current device, looked up once
// per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QLIN_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return QLIN_ERR_LAUNCH;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return QLIN_OK;
}

}  // namespace

extern "C" int qlin_forward_noalloc(int dtype, const void* x, int64_t ld_x, const void* wr, const void* wi,
                                    const void* wj, const void* wk, int64_t ld_w, const void* bias,
                                    const void* lora_a, const void* lora_b, int rank, float lora_scale,
                                    void* y, int64_t ld_y, int64_t M, int64_t K_g, int64_t N_g,
                                    void* stream) {
  size_t need = 0;
  int st = qlin_workspace_size(dtype, M, K_g, N_g, rank, &need);
  if (st != QLIN_OK) return st;
  // Problems whose scratch exceeds the fixed buffer are refused up front.
  if (need > (size_t)QLIN_NOALLOC_SCRATCH_BYTES) return QLIN_ERR_WORKSPACE;
  void* ws = nullptr;
  if (need > 0 && M > 0) {
    st = noalloc_scratch(&ws);
    if (st != QLIN_OK) return st;
  }
  // The scratch starts zero-filled (a device global) and only calls of this
  // entry point use it, so it meets QLIN_FLAG_ZEROED_WORKSPACE: its counter
  // bytes are zero between calls.  Every other byte a call reads was written
  // earlier in the same call.
  return qlin_forward_ex(dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank, lora_scale, y,
                         ld_y, M, K_g, N_g, ws, ws ? need : 0,
                         QLIN_ALGO_AUTO, ws ? QLIN_FLAG_ZEROED_WORKSPACE : 0, stream);
}
