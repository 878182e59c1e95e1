/*
 * qlin_b200.h -- C ABI of the B200 (sm_100a) quaternion linear forward.
 *
 * The quaternion linear layer replaces a real linear layer y = x W^T with
 * four real weight components Wr, Wi, Wj, Wk of shape [N_g, K_g] and the
 * Hamilton product per (output group, input group) pair.  Layout contract
 * (reference quaternion/packing.py:5-25): x[m, 4i+q] is component q (r,i,j,k)
 * of input quaternion i; y[m, 4o+a] is component a of output quaternion o;
 * W_c[o, i] is row-major with leading dimension ld_w.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream), returns a
 * status code, and never throws.  Work is enqueued asynchronously on the
 * given stream; nothing synchronises and nothing allocates device memory.
 */
#ifndef QLIN_B200_H
#define QLIN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types.  x, weights, bias, LoRA A/B and y all share one type. */
enum {
  QLIN_F32 = 0,  /* fp32 in, fp32 CUDA-core FMA accumulate, fp32 out        */
  QLIN_BF16 = 1, /* bf16 in, fp32 accumulate (tensor cores), one rounding out */
  QLIN_F16 = 2   /* fp16 in, fp32 accumulate (tensor cores), one rounding out */
};

/* Status codes. */
enum {
  QLIN_OK = 0,
  QLIN_ERR_SHAPE = 1,     /* bad dims or leading dims (reference: ValueError)   */
  QLIN_ERR_DTYPE = 2,     /* unsupported element type (reference: RuntimeError) */
  QLIN_ERR_ALIGN = 3,     /* pointer / leading-dim alignment not met by the path */
  QLIN_ERR_WORKSPACE = 4, /* workspace missing or smaller than qlin_workspace_size */
  QLIN_ERR_LAUNCH = 5,    /* a CUDA runtime call or kernel launch failed        */
  QLIN_ERR_DEVICE = 6,    /* the current device is not sm_100 (B200 class)      */
  QLIN_ERR_TIMEOUT = 7,   /* a bounded device-side wait ran out (see below)     */
  QLIN_ERR_ARG = 8,       /* null pointer or invalid option                     */
  QLIN_ERR_COLLECTIVE = 9 /* NCCL not loadable, or an NCCL call failed          */
};

/* Kernel selection for qlin_forward_ex (QLIN_ALGO_AUTO is what qlin_forward uses). */
enum {
  QLIN_ALGO_AUTO = 0,
  QLIN_ALGO_SIMT = 1,   /* CUDA-core tiled kernel: every dtype, every shape     */
  QLIN_ALGO_TC = 2,     /* TMA + tcgen05/TMEM kernel: bf16/f16, aligned shapes  */
  QLIN_ALGO_GEMV = 3    /* CUDA-core decode GEMV: bf16/f16, at most 4 tokens,
                           K_g a multiple of 8, LoRA rank <= 32 and a multiple
                           of 4 (then x and lora_a 16-byte aligned, ld_x a
                           multiple of 8); one launch without LoRA, two with
                           (the down-projection prologue, whose output lives in
                           the workspace); QLIN_ALGO_AUTO picks it for at most
                           2 tokens and at most one 8-quaternion CTA per SM    */
};

/*
 * Flags of qlin_forward_ex.
 *
 * QLIN_FLAG_STATIC_WEIGHTS: the caller guarantees that no work queued earlier
 * on the stream writes wr..wk, bias, lora_a or lora_b (inference with fixed
 * weights).  The kernels then start streaming the weights while the previous
 * kernel of the stream is still finishing (programmatic dependent launch);
 * x, the workspace and y are still only touched after it completed.
 * Without the flag every kernel waits for its predecessor before reading
 * any memory (plain stream order), overlapping only its launch and set-up.
 *
 * QLIN_FLAG_ZEROED_WORKSPACE: the workspace was zero-filled before its first
 * use and is only passed to calls of this library that are ordered with one
 * another (one stream).  Its first QLIN_WORKSPACE_COUNTER_BYTES bytes then
 * hold per-tile arrival counters that every call leaves at zero again, and a
 * K-split problem of at most 4 tokens sums its partial products inside the
 * main kernel (the last CTA of each tile to arrive) instead of in a separate
 * reduction kernel: one launch and one kernel hand-off fewer per call.  One
 * zeroed workspace may serve problems of any size: every non-zero
 * qlin_workspace_size() includes the counter bytes at its start, which no
 * other use of the workspace touches.
 *
 * QLIN_FLAG_NO_PAIR (comparisons and diagnostics): run prefill-sized
 * problems on the one-CTA tensor-core kernel (component planes from a
 * prologue kernel) instead of the CTA-pair kernel that QLIN_ALGO_AUTO and
 * QLIN_ALGO_TC otherwise use for them (more than 64 tokens, no LoRA, an even
 * number of output quaternions, ld_y a multiple of 8 and a 16-byte aligned y).
 *
 * QLIN_FLAG_NO_CLUSTER (comparisons and diagnostics): decode-sized
 * tensor-core problems (at most 16 tokens) sum their K split through the
 * workspace (the reduction kernel, or the last CTA of each tile on a zeroed
 * workspace) instead of the cluster reduce-scatter through distributed shared
 * memory that QLIN_ALGO_TC and QLIN_ALGO_AUTO otherwise use when the clusters
 * fit.
 */
enum {
  QLIN_FLAG_STATIC_WEIGHTS = 1,
  QLIN_FLAG_ZEROED_WORKSPACE = 2,
  QLIN_FLAG_NO_PAIR = 4,
  QLIN_FLAG_NO_CLUSTER = 8
};
#define QLIN_WORKSPACE_COUNTER_BYTES 4096u

/* Human-readable name of a status code (static storage). */
const char* qlin_status_string(int status);

/* ABI version (major * 100 + minor). */
int qlin_abi_version(void);

/*
 * Bytes of device workspace qlin_forward needs for this problem (0 for some
 * paths).  rank = LoRA rank (0 = no LoRA).  The workspace holds the planar
 * copy of x (M > 64), the LoRA down projection and the fp32 partial sums of
 * a K split; it is only used during the call's kernels and needs no
 * initialisation, so one buffer can be reused by calls on the same stream.
 */
int qlin_workspace_size(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank,
                        size_t* bytes);

/*
 * y = QuaternionLinear(x) (+ bias) (+ lora_scale * ((x A^T) B^T)).
 *
 * Replaces, for the device path:
 *   quaternion/linear.py:41-72    quaternion_linear(x, wr, wi, wj, wk)
 *   quaternion/linear.py:120-124  QuaternionLinear.forward (bias added)
 *   quaternion/planar.py:39-61    quaternion_linear_naive   (same math, K1)
 *   quaternion/planar.py:100-129  quaternion_linear_planar  (same math, K2)
 *   quaternion/lora.py:60-63      LoRAQuaternionLinear.forward (fused residual)
 *   kernels/cuda/quaternion_linear.cu:117-159  quaternion_linear_forward (K4)
 *   kernels/triton/quaternion.py:104-133       _launch (K3)
 *
 *   x      [M, 4*K_g], leading dimension ld_x (elements, >= 4*K_g)
 *   wr..wk [N_g, K_g] each, leading dimension ld_w (>= K_g)
 *   bias   [4*N_g] or NULL
 *   lora_a [rank, 4*K_g] contiguous, lora_b [4*N_g, rank] contiguous, or both
 *          NULL with rank = 0; lora_scale = alpha / rank
 *   y      [M, 4*N_g], leading dimension ld_y (>= 4*N_g); must not alias x
 *   workspace: device buffer of at least qlin_workspace_size() bytes,
 *          256-byte aligned (may be NULL when that size is 0)
 * M = 0 is a no-op.  Accumulation is fp32; bf16/f16 outputs are rounded
 * once, after bias and LoRA are added.
 */
int qlin_forward(int dtype,
                 const void* x, int64_t ld_x,
                 const void* wr, const void* wi, const void* wj, const void* wk,
                 int64_t ld_w,
                 const void* bias,
                 const void* lora_a, const void* lora_b, int rank, float lora_scale,
                 void* y, int64_t ld_y,
                 int64_t M, int64_t K_g, int64_t N_g,
                 void* workspace, size_t workspace_bytes,
                 void* stream);

/* qlin_forward with an explicit kernel choice (QLIN_ALGO_*; tests run both
 * device paths on the same inputs) and flags (QLIN_FLAG_*).  QLIN_ALGO_TC
 * returns QLIN_ERR_ALIGN when the shape or pointers do not meet its TMA
 * rules. */
int qlin_forward_ex(int dtype,
                    const void* x, int64_t ld_x,
                    const void* wr, const void* wi, const void* wj, const void* wk,
                    int64_t ld_w,
                    const void* bias,
                    const void* lora_a, const void* lora_b, int rank, float lora_scale,
                    void* y, int64_t ld_y,
                    int64_t M, int64_t K_g, int64_t N_g,
                    void* workspace, size_t workspace_bytes,
                    int algo, int flags, void* stream);

/* qlin_plan's algo for the tensor-core path run on the CTA-pair kernel
 * (persistent, two SMs per tile, 2-SM tcgen05 UMMA); not an input value. */
#define QLIN_PLAN_TC_PAIR 4

/*
 * qlin_forward with the packed weight cache (no reference counterpart: the
 * reference keeps only the four component tensors, quaternion/linear.py:101-104).
 *
 *   wq     [N_g][ld_wq][4]: wq[o][i][p] = W_p[o][i], all four components of a
 *          weight quaternion side by side (the layout of x rows); ld_wq in
 *          quaternions, even; 16-byte aligned; bf16/f16 only; K_g a multiple
 *          of 8 (otherwise the planar weights are used)
 *   wr..wk the planar components as in qlin_forward, or all four NULL
 * The kernels that read the packed buffer take it: the decode GEMV (at most
 * 2 tokens) reads one address stream per output row instead of four, and the
 * CTA-pair prefill kernel's builder warps get all four components of an input
 * quaternion from one 8-byte piece.  Every other path reads the planar
 * weights; without them such a problem returns QLIN_ERR_ALIGN.  Results equal
 * qlin_forward's on the same weights (same kernels' arithmetic).
 * Other arguments as qlin_forward_ex with QLIN_ALGO_AUTO.
 */
int qlin_forward_packed(int dtype,
                        const void* x, int64_t ld_x,
                        const void* wq, int64_t ld_wq,
                        const void* wr, const void* wi, const void* wj, const void* wk,
                        int64_t ld_w,
                        const void* bias,
                        const void* lora_a, const void* lora_b, int rank, float lora_scale,
                        void* y, int64_t ld_y,
                        int64_t M, int64_t K_g, int64_t N_g,
                        void* workspace, size_t workspace_bytes,
                        int flags, void* stream);

/*
 * Launch plan qlin_forward_ex uses for this problem with these flags on the
 * current device (diagnostics; no reference counterpart; flags 0 is
 * qlin_forward's plan).  Fills every non-null output:
 * algo (QLIN_ALGO_* or QLIN_PLAN_TC_PAIR, assuming aligned pointers), tokens per tensor-core tile,
 * K split (CTAs sharing one output tile), kernel launches per call, and how
 * many CTAs of the tensor-core kernel the device keeps resident at once.
 */
int qlin_plan(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank, int flags, int* algo,
              int* tile_tokens, int* split_k, int* launches, int* resident_ctas);

/*
 * One rank's shard of a layer column-partitioned along out/4 over `world`
 * GPUs of one box, fused with the all-gather of the outputs (replaces the
 * shard-then-NCCL-all-gather path; the reference has no distributed path).
 *
 * This rank computes output quaternion rows [N_g] of its shard (wr..wk,
 * bias and lora_b hold the shard's rows; x and lora_a are replicated) and
 * its epilogue stores every output both into its own full output and, over
 * NVLink, into every other rank's, at columns [col_offset, col_offset+4*N_g):
 *   outs        host array [world] of device pointers, as mapped in this
 *               process (CUDA IPC), to every rank's full output [M, ld_out]
 *               (outs[world_rank] is this rank's own);
 *   flag_arrays host array [world] of device pointers to every rank's
 *               barrier flags, unsigned[2 * world], zero before the first call;
 *   epoch_word  this rank's two call counters, unsigned[2] (device, zero
 *               before the first call).
 * Two one-warp barrier kernels bracket the shard kernel: the entry barrier
 * keeps every rank from storing into a peer's output before that peer has
 * finished the work it queued on its stream after the previous call (for
 * example reading or copying that output); after the exit barrier every
 * rank's full output holds all ranks' columns.  Every rank must make the
 * same sequence of calls.  16-bit types, tensor-core path only; waits are
 * bounded (2 s; QLIN_ERR_TIMEOUT via qlin_get_device_error, after which the
 * outputs of that call are undefined).  The other arguments are those of
 * qlin_forward_ex (algo is the tensor-core kernel).
 */
int qlin_forward_allgather(int dtype,
                           const void* x, int64_t ld_x,
                           const void* wr, const void* wi, const void* wj, const void* wk,
                           int64_t ld_w,
                           const void* bias,
                           const void* lora_a, const void* lora_b, int rank, float lora_scale,
                           int64_t M, int64_t K_g, int64_t N_g,
                           void* workspace, size_t workspace_bytes, int flags,
                           int world, int world_rank,
                           void* const* outs, int64_t ld_out, int64_t col_offset,
                           unsigned* const* flag_arrays, unsigned* epoch_word,
                           void* stream);

/*
 * qlin_forward_allgather with the full output bound to an NVLink multicast
 * object (e.g. a symmetric-memory buffer): `out` is this rank's full output
 * [M, ld_out] and out_mc the multicast address of the same buffer on every
 * rank.  Each output piece of this rank's columns is stored once through
 * out_mc (multimem.st): NVSwitch writes it into every rank's output, this
 * rank's included, so each rank sends its columns over NVLink once instead
 * of once per peer.  The entry and exit flag barriers are those of
 * qlin_forward_allgather (flag_arrays[2 * world], epoch_word[2]).
 */
int qlin_forward_allgather_mc(int dtype,
                              const void* x, int64_t ld_x,
                              const void* wr, const void* wi, const void* wj, const void* wk,
                              int64_t ld_w,
                              const void* bias,
                              const void* lora_a, const void* lora_b, int rank, float lora_scale,
                              int64_t M, int64_t K_g, int64_t N_g,
                              void* workspace, size_t workspace_bytes, int flags,
                              int world, int world_rank,
                              void* out, void* out_mc, int64_t ld_out, int64_t col_offset,
                              unsigned* const* flag_arrays, unsigned* epoch_word,
                              void* stream);

/*
 * qlin_forward_ex with the input and output in host memory (no reference
 * counterpart: the reference's CPU callers hand over host tensors).  x_host
 * [M, ld_x] is copied to the device, the layer runs, and y [M, ld_y] is
 * copied back to y_host, all enqueued on `stream` in that order; y_host
 * holds the result once the stream has reached that point (synchronise the
 * stream or an event).  Host buffers should be page-locked (cudaHostAlloc /
 * cudaHostRegister) for the copies to be asynchronous.  For decode-sized
 * page-locked buffers (at most 64 KB, rows of whole 16-byte words) x comes
 * in by a small kernel and the layer's kernels store y straight into the
 * host buffer through its device mapping; otherwise copy-engine transfers.  Weights, bias and
 * LoRA stay device pointers.  workspace (device): at least
 * qlin_host_workspace_size() bytes -- the staged x and y, then the
 * workspace of qlin_forward_ex, which QLIN_FLAG_ZEROED_WORKSPACE refers to
 * (zero-fill the whole buffer once).
 */
int qlin_forward_host(int dtype,
                      const void* x_host, int64_t ld_x,
                      const void* wr, const void* wi, const void* wj, const void* wk,
                      int64_t ld_w,
                      const void* bias,
                      const void* lora_a, const void* lora_b, int rank, float lora_scale,
                      void* y_host, int64_t ld_y,
                      int64_t M, int64_t K_g, int64_t N_g,
                      void* workspace, size_t workspace_bytes,
                      int algo, int flags, void* stream);
int qlin_host_workspace_size(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank, size_t* bytes);

/*
 * Column-partitioned layer over NCCL (no reference counterpart: the exchange
 * of a layer whose output quaternions are split over `world` GPUs), for
 * hosts that hold an NCCL communicator but no peer-mapped output buffers.
 *
 * This process is rank world_rank of nccl_comm (an ncclComm_t of `world`
 * ranks on the current device).  Every rank passes its own slice of the
 * layer: wr..wk [N_g, ld_w] are its output quaternions [world_rank * N_g,
 * (world_rank + 1) * N_g), bias [4 N_g] and lora_b [4 N_g, rank] the same
 * rows; x and lora_a are the full inputs, equal on every rank.  y [M, ld_y]
 * with ld_y >= world * 4 * N_g receives every rank's columns, rank r's at
 * column offset r * 4 * N_g (the full layer's output on every rank).
 *
 * On `stream`: this rank's columns by the single-GPU kernels (for M == 1
 * straight into y, else into the workspace), one ncclAllGather of M * 4 * N_g
 * elements per rank, and for M > 1 one kernel that places the gathered
 * column blocks into y's rows.  workspace: at least
 * qlin_sharded_workspace_size() bytes, used as qlin_forward_ex's with the
 * same flags.  The NCCL library is the one the process has already loaded,
 * else libnccl.so.2; QLIN_ERR_COLLECTIVE when neither is found or an NCCL
 * call fails.  Capturable in a CUDA graph when NCCL's own calls are.
 */
int qlin_sharded_fwd(int dtype,
                     const void* x, int64_t ld_x,
                     const void* wr, const void* wi, const void* wj, const void* wk,
                     int64_t ld_w,
                     const void* bias,
                     const void* lora_a, const void* lora_b, int rank, float lora_scale,
                     void* y, int64_t ld_y,
                     int64_t M, int64_t K_g, int64_t N_g,
                     void* workspace, size_t workspace_bytes, int flags,
                     void* nccl_comm, int world, int world_rank,
                     void* stream);
int qlin_sharded_workspace_size(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank, int world,
                                size_t* bytes);

/*
 * NCCL bootstrap for callers of qlin_sharded_fwd that have no NCCL binding of
 * their own (the same library it calls): qlin_nccl_unique_id writes a
 * 128-byte ncclUniqueId, which the caller sends to every rank by its own
 * means; qlin_nccl_comm_init creates this rank's communicator on the current
 * device (blocking until all `world` ranks joined, as ncclCommInitRank);
 * qlin_nccl_comm_destroy releases it.
 */
int qlin_nccl_unique_id(void* id);
int qlin_nccl_comm_init(void** comm, int world, const void* id, int world_rank);
int qlin_nccl_comm_destroy(void* comm);

/*
 * Buffers shared between the processes of a column-partitioned layer (no
 * reference counterpart; plumbing of qlin_forward_allgather).
 * qlin_ipc_alloc allocates `bytes` of zero-filled device memory on the
 * current device with plain cudaMalloc (so that its CUDA IPC handle exists
 * whatever allocator the host framework uses) and writes the 64-byte
 * cudaIpcMemHandle to `handle`; qlin_ipc_free releases it.  qlin_ipc_open
 * maps another process's buffer, given its handle and a byte offset into
 * it, for the current device (peer access enabled lazily) and returns the
 * address of base + offset; qlin_ipc_close takes the mapped base.
 */
int qlin_ipc_alloc(size_t bytes, void** out, void* handle);
int qlin_ipc_free(void* p);
int qlin_ipc_open(const void* handle, int64_t offset, void** out);
int qlin_ipc_close(void* base);

/* Which algorithm qlin_forward would pick for this problem (QLIN_ALGO_*). */
int qlin_select_algo(int dtype, int64_t M, int64_t K_g, int64_t N_g, int rank);

/*
 * Allocation-free variant of qlin_forward (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory where they run the layer
 * (code that must not call cudaMalloc mid-stream because it can synchronise
 * the device, framework plugins that are handed only their input and output
 * buffers, runtimes that forbid allocation after start-up).  Same arguments
 * and kernels as qlin_forward, but no workspace: the scratch comes from a
 * fixed buffer of QLIN_NOALLOC_SCRATCH_BYTES compiled into the library, which
 * every GPU that loads the library holds until the process exits.
 *
 *  - A problem is accepted when qlin_workspace_size() for it is at most
 *    QLIN_NOALLOC_SCRATCH_BYTES (8 MiB; decode-sized layers fit), and refused
 *    with QLIN_ERR_WORKSPACE before any device work otherwise.  Ask
 *    qlin_workspace_size() rather than estimating: the scratch holds the
 *    planar copy of x (M * in_features elements when M > 64), the LoRA down
 *    projection, fp32 split-K partials and 4096 counter bytes.
 *  - The first call on a device looks up the buffer's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.
 *  - All calls on a device share the one buffer.  It starts zero-filled and
 *    only this entry point uses it, so calls run as with
 *    QLIN_FLAG_ZEROED_WORKSPACE (decode-sized K splits summed inside the
 *    main kernel; its counter bytes are back at zero after every call).
 *    Calls that overlap on the GPU -- on different streams, or from
 *    different threads -- race on it; serialise them (one stream, or events
 *    between streams).
 * Nothing is allocated: no cudaMalloc, no cudaFree, no allocating library call.
 */
#define QLIN_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
int qlin_forward_noalloc(int dtype,
                         const void* x, int64_t ld_x,
                         const void* wr, const void* wi, const void* wj, const void* wk,
                         int64_t ld_w,
                         const void* bias,
                         const void* lora_a, const void* lora_b, int rank, float lora_scale,
                         void* y, int64_t ld_y,
                         int64_t M, int64_t K_g, int64_t N_g,
                         void* stream);

/*
 * Device-side error word.  Every wait inside the kernels (TMA arrival, MMA
 * completion) is bounded; a wait that runs out records QLIN_ERR_TIMEOUT here
 * and the kernel returns without further work instead of hanging the GPU.
 * qlin_get_device_error synchronises `stream`, reads the word for the
 * current device and clears it when `clear` is non-zero.
 */
int qlin_get_device_error(void* stream, int clear, int* device_status);

/*
 * Column gather for the column-partitioned layer: src holds G shards
 * [G, M, n_shard] (the layout an all-gather of per-rank [M, n_shard]
 * outputs produces); dst receives [M, G * n_shard] with leading dimension
 * ld_dst.  Element size = that of dtype.
 */
int qlin_gather_columns(int dtype, const void* src, void* dst, int64_t G, int64_t M,
                        int64_t n_shard, int64_t ld_dst, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QLIN_B200_H */
