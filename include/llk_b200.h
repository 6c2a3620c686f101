/*
 * llk_b200.h -- C ABI of the B200 (sm_100a) backend for DSLCompiler's fused
 * SwiGLU and micro.mma matmul path.
 *
 * Everything here is plain C: pointers, sizes and integer status codes; no
 * CUDA, torch or C++ types cross this boundary (streams are passed as
 * `void *` holding a cudaStream_t).  Each declaration names the reference
 * interface it replaces, by file:line inside the DSLCompiler project.
 *
 * Data contract (the llk.fused_swiglu op, include/LLK/Dialect/LLKOps.td:13-67):
 *   X[M,K], Wg[K,N], Wu[K,N] bf16, row-major, strides in ELEMENTS
 *   (runtime/PackedWeights.cpp:21 uses stride0 as an element count);
 *   Y[M,N] bf16 (or f32 through llk_swiglu_ex);  f32 accumulation;
 *   Y = SiLU(X*Wg) (.) (X*Wu)   (lib/Transforms/FuseDoubleContraction.cpp:119-199).
 *
 * Pointers may be device memory (the call is then asynchronous on the given
 * stream) or host memory (the call stages the data through the device and
 * returns when Y is back on the host, like the reference's synchronous
 * CPU kernel).  There is no CPU fallback: without a usable sm_100 GPU every
 * entry point fails with LLK_ERR_DEVICE.
 */
#ifndef LLK_B200_H
#define LLK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- data descriptors (layouts identical to the reference) ------------ */

/* include/LLK/Runtime/JitCache.h:30-36 */
typedef struct Tensor2D {
  void *data;
  int64_t dim0;
  int64_t dim1;
  int64_t stride0;
  int64_t stride1;
} Tensor2D;

/* include/LLK/Runtime/JitCache.h:42-50 (56 bytes, MLIR memref<MxN> ABI) */
typedef struct MemRef2D {
  void *allocated;
  void *aligned;
  int64_t offset;
  int64_t size0;
  int64_t size1;
  int64_t stride0;
  int64_t stride1;
} MemRef2D;

/* include/LLK/Runtime/JitCache.h:59-62.  `scratch` may point at DEVICE
 * memory the library may use as workspace (split-K partial sums, work
 * counters); NULL lets the library use its own per-device workspace.
 *
 * Concurrency: the library workspace is one buffer per device.  Calls with
 * device buffers return once their kernel is queued, so two calls that rely
 * on it (decode-shaped SwiGLU, or prefill over 12 or more waves of tiles)
 * and may overlap on the GPU -- different streams, or threads without
 * ordering between them -- race on its counters and partial sums.  Serialise
 * such calls per device (one stream, or events), or give each concurrent
 * caller its own `scratch`.  After a kernel gives up a bounded wait
 * (LLK_ERR_TIMEOUT), llk_synchronize clears the workspace as well as the
 * status word, so later calls start from zeroed counters. */
typedef struct KernelContext {
  void *scratch;
  size_t scratch_size;
} KernelContext;

/* ---- status codes ------------------------------------------------------ */
/* The reference kernel returns void and reports compile errors through
 * llvm::Expected (runtime/JitCache.cpp:200-235); device launches need
 * run-time codes. */
enum llk_status_code {
  LLK_OK = 0,
  LLK_ERR_SHAPE = 1,       /* dims inconsistent (LLKOps.cpp:42-83 rules) */
  LLK_ERR_ALIGN = 2,       /* non-unit inner stride, misaligned pointer */
  LLK_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  LLK_ERR_NCCL = 4,        /* a collective failed */
  LLK_ERR_TIMEOUT = 5,     /* a device-side wait gave up (bounded waits) */
  LLK_ERR_ARG = 6,         /* NULL pointer or bad enum value */
  LLK_ERR_DEVICE = 7,      /* no sm_100 device, or library not usable */
  LLK_ERR_UNSUPPORTED = 8, /* valid request this backend does not do */
  LLK_ERR_NOMEM = 9,       /* scratch too small / allocation failed */
  LLK_ERR_NOT_FOUND = 10   /* cache lookup without an entry */
};

/* include/LLK/Runtime/KernelKey.h:23 (DType) */
enum llk_dtype { LLK_DTYPE_BF16 = 0, LLK_DTYPE_FP16 = 1, LLK_DTYPE_FP32 = 2 };

/* Which kernel family serves a call (KernelKey.isa / micro.kernel
 * `candidate` analogue).  AUTO picks by shape. */
enum llk_variant {
  LLK_VARIANT_AUTO = 0,
  LLK_VARIANT_TC = 1,     /* tcgen05 + TMA tiled kernel (prefill / GEMM) */
  LLK_VARIANT_DECODE = 2, /* small-M weight-streaming kernel */
  LLK_VARIANT_SIMT = 3    /* CUDA-core kernel for any stride/alignment */
};

/* The SiLU epilogue's numerics (include/LLK/Runtime/KernelKey.h:39 MathMode,
 * the op's math_mode attribute).  STRICT: sigmoid = 1 / (1 + exp(-g)) with
 * an accurate exp and an IEEE-rounded division, the fused lowering's
 * sequence (lib/Transforms/FuseDoubleContraction.cpp:189-196).  The fast
 * modes use the hardware's approximate exp and division (about 2 ulp each);
 * BOUNDED_FAST and UNSAFE_FAST run the same kernels here. */
enum llk_math_mode { LLK_MATH_STRICT = 0, LLK_MATH_BOUNDED_FAST = 1, LLK_MATH_UNSAFE_FAST = 2 };

/* GPU-side call options, carried beside (not inside) KernelContext so that
 * struct keeps the reference's 16-byte layout.  Zero-filled = current
 * device, default stream, bf16 Y, automatic kernel choice, strict math. */
typedef struct llk_gpu_context {
  int device;      /* CUDA ordinal the pointers live on; -1 = current */
  void *stream;    /* cudaStream_t; NULL = legacy default stream */
  int y_dtype;     /* enum llk_dtype: BF16 (op contract) or FP32 */
  int variant;     /* enum llk_variant */
  int math_mode;   /* enum llk_math_mode (SwiGLU epilogue; matmul ignores it) */
  int reserved[3]; /* must be zero */
} llk_gpu_context;

/* ---- entry points ------------------------------------------------------ */

/* The documented public kernel symbol:
 *   extern "C" void llk_swiglu(const Tensor2D*, const Tensor2D*,
 *                              const Tensor2D*, Tensor2D*, KernelContext*)
 * (docs/design/m1-scalar-pipeline.md:177-197).  Y is bf16.  Returns void
 * like the reference; the outcome is available from llk_last_status(). */
void llk_swiglu(const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, Tensor2D *y, KernelContext *ctx);

/* Same operation with GPU options and a status result (gpu may be NULL). */
int llk_swiglu_ex(const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, Tensor2D *y, KernelContext *ctx,
                  const llk_gpu_context *gpu);

/* The JIT'd kernel calling convention JitCache::KernelFn
 * (include/LLK/Runtime/JitCache.h:80-81): five MemRef2D* = x, wg, wu, init,
 * result.  `init` is ignored (the fused op overwrites; LLKOps.td:29-41);
 * result is bf16.  Outcome via llk_last_status(). */
void llk_swiglu_memref(MemRef2D *x, MemRef2D *wg, MemRef2D *wu, MemRef2D *init, MemRef2D *result);

/* micro.mma / linalg.matmul: C[M,N] (f32) = (accumulate ? C : 0) + A*B with
 * A[M,K], B[K,N] bf16 and f32 accumulation (micro.mma acc += lhs x rhs,
 * include/LLK/Dialect/Micro/MicroOps.td:196-222, verifier
 * lib/Dialect/Micro/MicroOps.cpp:246-291). */
int llk_matmul(const Tensor2D *a, const Tensor2D *b, Tensor2D *c, int accumulate, KernelContext *ctx,
               const llk_gpu_context *gpu);

/* ---- llk.rope / llk.attention (include/LLK/Dialect/LLKOps.td:69-131) -----
 * The reference's other two LLK ops, lowered by
 * lib/Conversion/LLKToLinalg/LLKToLinalg.cpp:162-615.  All arrays are
 * contiguous row-major; f32 data, i64 position ids.  Host arrays are staged
 * through the device and the call returns with the result on the host;
 * device arrays must live on the call's device (asynchronous on
 * gpu->stream).  gpu->math_mode STRICT uses accurate cos / sin / exp (the
 * ops' math.cos / math.sin / math.exp), the fast modes the hardware's
 * approximations. */

/* RoPE: y[b,h,p,2i]   = x[..,2i] * c - x[..,2i+1] * s,
 *       y[b,h,p,2i+1] = x[..,2i+1] * c + x[..,2i] * s,
 * c, s = cos / sin of (f32) position_ids[p] * theta^(-2i/D) (computed in
 * f64).  x, y: [B, H, L, D] (y may equal x); position_ids: [L]; D even
 * (else LLK_ERR_SHAPE), theta > 0.  The (cos, sin) table, L * D/2 * 8
 * bytes, is built in the library's per-device workspace (grown with
 * cudaMalloc on first use; calls on one device are serialised as for the
 * other workspace users, see KernelContext). */
int llk_rope(const float *x, const int64_t *position_ids, float *y, int64_t B, int64_t H, int64_t L, int64_t D,
             double theta, const llk_gpu_context *gpu);

/* Attention, destination-passing like the op (its `init` operand):
 *   o[b,h,i,:] += sum_j softmax_j(scale * q[b,h,i,:] . k[b,h,j,:]) v[b,h,j,:],
 * with keys j > i masked out when causal.  q, o: [B, H, Lq, D]; k, v:
 * [B, H, Lk, D]; o must not alias q, k or v (LLK_ERR_ARG).  With Lk = 0, o
 * keeps its values.  B * H <= 65535. */
int llk_attention(const float *q, const float *k, const float *v, float *o, int64_t B, int64_t H, int64_t Lq,
                  int64_t Lk, int64_t D, float scale, int causal, const llk_gpu_context *gpu);

/* Status of the last call on this host thread (llk_swiglu, _memref). */
int llk_last_status(void);
const char *llk_status_string(int status);

/* Wait for `stream` (cudaStream_t, NULL = default) on `device` (-1 =
 * current) and return LLK_ERR_TIMEOUT if any kernel launched by this
 * library on that device since the last check gave up a bounded wait, else
 * LLK_OK; clears the device's error word. */
int llk_synchronize(int device, void *stream);

/* Diagnostic: launches a kernel whose bounded device-side wait is made to
 * expire after `limit_ns` (nothing ever arrives on its barrier), waits for
 * it and returns the device status -- LLK_ERR_TIMEOUT when the timeout path
 * works.  No counterpart in the reference (its waits are unbounded,
 * runtime/ThreadPool.cpp:96-103); it lets the failure path be tested on a
 * GPU without a fault or a hang. */
int llk_diag_timeout_probe(int device, int64_t limit_ns);

/* Diagnostic: the strict SwiGLU epilogue computes 1 / (1 + e^-g) with its
 * own correctly rounded reciprocal (Markstein's method) instead of the
 * general IEEE division; this counts, into *mismatches, the floats with bit
 * patterns in [lo_bits, hi_bits) on which it differs from CUDA's correctly
 * rounded reciprocal.  0 over [0x3f800000, 0x7f800000) (every finite b >= 1)
 * shows the epilogue equals the division.  No counterpart in the reference. */
int llk_diag_reciprocal_check(int device, uint32_t lo_bits, uint32_t hi_bits, uint64_t *mismatches);

/* Diagnostic (host only, no GPU needed): the CTA-pair kernel's work split
 * for a problem (swiglu != 0: fused SwiGLU, 128 Y columns per pair tile;
 * else matmul, 256) on `pairs` CTA pairs, as the launch computes it --
 * whole-tile waves, then the leftover tiles cut along N (tail_split 1, 2, 4)
 * or along K (-s: s parts; 0 = the launch's own choice).  Writes up to
 * max_items items of 9 int32 each: {pair (-1 when dynamic), row tile, column
 * tile, first column, width, first k-block, end k-block, K part, K parts},
 * and the item count, the pairs launched, the K split (0 = none) and the
 * column split chosen.  No counterpart in the reference. */
int llk_diag_pair_schedule(int swiglu, int64_t M, int64_t N, int64_t K, int pairs, int tail_split, int dynamic,
                           int32_t *items, int max_items, int *n_items, int *n_pairs, int *ksplit,
                           int *tail_split_out);

/* ---- decode without device allocation -------------------------------- */

/* Size of the fixed device scratch array behind llk_swiglu_decode_noalloc
 * (16 MiB; every GPU that loads the library holds it until exit), and the
 * widest N it serves (its per-tile arrival counters: one int per 128
 * columns, 65536 of them). */
#define LLK_DECODE_NOALLOC_SCRATCH_BYTES (16u << 20)
#define LLK_DECODE_NOALLOC_MAX_N (65536ll * 128)

/* The small-M (decode) fused SwiGLU for callers that cannot allocate device
 * memory: code whose GPU memory is owned by another allocator (e.g. a
 * framework's caching allocator that has reserved the HBM, where a raw
 * cudaMalloc would fail or fragment it) or latency-critical loops where
 * cudaMalloc/cudaFree would add host round trips and implicit device-wide
 * synchronisation.  No counterpart in the reference (its CPU kernel takes
 * scratch through KernelContext).
 *
 * It runs the same decode kernel as llk_swiglu_ex (variant DECODE), but its
 * split-K workspace is a fixed file-scope device array of
 * LLK_DECODE_NOALLOC_SCRATCH_BYTES, so the call allocates nothing: no
 * cudaMalloc/cudaFree, no library allocator.  The caller passes inputs and
 * outputs in DEVICE memory of the call's device (or managed memory); host
 * buffers and other GPUs' buffers are refused with LLK_ERR_ARG, as staging
 * them would need device memory.  Limits: 1 <= M <= 128 (else
 * LLK_ERR_UNSUPPORTED) and N <= LLK_DECODE_NOALLOC_MAX_N (else
 * LLK_ERR_NOMEM: the array holds the counters of at most that many
 * columns).  The workspace a launch needs is 264 KB (8 KB + 256 KB) of counters
 * plus, when a stream-K grid has CTAs sharing a column tile, 4096 * Mp bytes
 * per CTA (Mp = M rounded up to 16, 32, 64 or 128); when that would not fit,
 * the call runs on fewer CTAs instead (possible only for M > 32).
 * Rows of X/Wg/Wu need 16-byte aligned starts and pitches, Y a start
 * aligned to its element size (else LLK_ERR_ALIGN).  Y is bf16, or f32
 * when gpu->y_dtype == LLK_DTYPE_FP32.
 *
 * The first call on a device performs a set-up with that device current (it
 * looks up the array's device address with cudaGetSymbolAddress); make that
 * first call before any stream capture.  A set-up that fails is not
 * remembered: the next call tries again.  The caller's current device is
 * restored before the call returns.  Every call shares the one array and it
 * keeps the last call's contents: each call clears the counters that must
 * start at zero.  Calls that overlap on the GPU (different streams, or
 * threads without ordering) race on the array and corrupt each other's
 * results -- serialise them.
 *
 * device_status, if not NULL, is a device int that receives LLK_ERR_TIMEOUT
 * when a bounded wait in the kernel gives up (the call does not clear it).
 * Asynchronous on gpu->stream (NULL gpu: current device, default stream). */
int llk_swiglu_decode_noalloc(const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, Tensor2D *y,
                              int *device_status, const llk_gpu_context *gpu);

/* ---- packed weights (runtime/PackedWeights.cpp:5-37, PackedWeights.h:13-49,
 *      and the L4 weight cache of include/LLK/Runtime/JitCache.h:143-146) --- */

/* Opaque device-resident copy of Wg/Wu laid out for the kernels' TMA boxes.
 * Built once; the weights are then not read from the caller again, so a
 * caller that changes its weights calls llk_repack (PackedWeights.h:49). */
typedef struct llk_packed_weights llk_packed_weights;

int llk_pack_weights(const Tensor2D *wg, const Tensor2D *wu, const llk_gpu_context *gpu, llk_packed_weights **out);
int llk_repack(llk_packed_weights *pw, const Tensor2D *wg, const Tensor2D *wu, const llk_gpu_context *gpu);
void llk_packed_weights_free(llk_packed_weights *pw);
/* K, N and the device bytes held. */
int llk_packed_weights_info(const llk_packed_weights *pw, int64_t *K, int64_t *N, int64_t *bytes);
int llk_swiglu_packed(const Tensor2D *x, const llk_packed_weights *pw, Tensor2D *y, KernelContext *ctx,
                      const llk_gpu_context *gpu);

/* Device layout of a packed pair: for each of Wg and Wu, ceil(N/box_n)
 * slabs of [K][box_n] bf16 (slab s holds columns s*box_n ..), each slab
 * contiguous, so one TMA box of box_n x box_k elements is one contiguous
 * 8 KB block.  Pointers are device pointers on *device. */
typedef struct llk_packed_layout {
  void *wg;
  void *wu;
  int device;
  int box_n; /* 64 columns per slab (BN) */
  int box_k; /* 64 rows of K per TMA box / pipeline stage (BK) */
  int64_t slab_stride_bytes; /* K * box_n * 2 */
} llk_packed_layout;

int llk_packed_weights_layout(const llk_packed_weights *pw, llk_packed_layout *out);

/* ---- L4 packed-weight cache (JitCache.h:138-146; WeightKey,
 *      KernelKey.h:112-124) ---------------------------------------------
 * Device-resident packed pairs keyed by WeightKey, LRU-evicted beyond the
 * level-4 maximum.  Handles are reference counted: llk_pack_weights and
 * every hit of llk_lookup_packed_weights hand the caller one reference,
 * released with llk_packed_weights_free; the cache holds its own reference
 * from llk_insert_packed_weights until the entry is evicted, replaced or
 * cleared, so a handle a caller looked up stays valid until the caller
 * frees it.  (The reference's L4 stores a serialised host blob; this one
 * stores the device copy the kernels read.) */
typedef struct llk_weight_key {
  const void *weight_ptr; /* the caller's Wg data pointer */
  uint64_t shape_hash;    /* see llk_weight_key_for */
  int64_t BK;             /* box rows of K (64) */
  int64_t BN;             /* slab width (64) */
} llk_weight_key;

/* Key for the pair (wg, wu): weight_ptr = wg->data; shape_hash mixes K, N,
 * both row strides and wu->data (two pairs sharing Wg but not Wu differ);
 * BK = BN = 64. */
int llk_weight_key_for(const Tensor2D *wg, const Tensor2D *wu, llk_weight_key *out);
/* LLK_OK and a new reference in *out on a hit; LLK_ERR_NOT_FOUND on a miss. */
int llk_lookup_packed_weights(const llk_weight_key *key, llk_packed_weights **out);
/* The cache takes its own reference (the caller keeps theirs). */
int llk_insert_packed_weights(const llk_weight_key *key, llk_packed_weights *pw);

/* ---- column sharding (multi-GPU) --------------------------------------- */

/* Columns [begin, end) of an N-column output owned by shard `index` of
 * `n_shards` when 128-column tiles are dealt out as evenly as possible
 * (earlier shards take the remainder).  Returns LLK_ERR_ARG on bad input. */
int llk_shard_columns(int64_t N, int n_shards, int index, int64_t *begin, int64_t *end);

/* After an all-gather of equal-width (padded) column shards, shard-major
 * `shards` = [n_shards][M][width] (device, elem_bytes 2 = bf16 or 4 = f32)
 * holds shard s's columns [begins[s], begins[s+1]) in its first
 * begins[s+1]-begins[s] columns; writes them into row-major device Y
 * (row stride ldy elements).  begins: host array of n_shards + 1 offsets,
 * n_shards <= 64.  Asynchronous on gpu->stream.  No counterpart in the
 * reference (it has no multi-device path). */
int llk_gather_columns(const void *shards, int n_shards, int64_t M, int64_t width, const int64_t *begins, void *y,
                       int64_t ldy, int elem_bytes, const llk_gpu_context *gpu);

/* ---- column-parallel SwiGLU with the all-gather fused in ----------------
 * One process per GPU, n_ranks <= 8 on one node.  Each rank owns the
 * columns llk_shard_columns(N, n_ranks, rank) of Wg/Wu and a replica of X;
 * llk_swiglu_column_parallel computes those columns and the CTA-pair
 * kernel's epilogue stores every finished chunk into EVERY rank's Y over
 * NVLink (peer stores; the 1-CTA and decode kernels used for M <= 128 copy
 * their columns with the copy engines instead), so when the call's work
 * completes in stream order, this rank's group Y holds the whole Y[M, N]
 * (row-major, row stride N, bf16 or f32 per gpu->y_dtype).  This replaces
 * compute + ncclAllGather + relayout (the reference has no multi-device
 * path).  Set-up, once per group:
 *   1. every rank: llk_peer_group_create -> a handle of LLK_IPC_HANDLE_BYTES;
 *   2. exchange the handles over any host channel (rank order);
 *   3. every rank: llk_peer_group_connect with all n_ranks handles.
 * Every rank must make the same sequence of calls.  Calls alternate
 * between two Y buffers and end with a device-side barrier over the group
 * (bounded: 2 s; a rank that never arrives makes the others report
 * LLK_ERR_TIMEOUT through llk_synchronize), so a call never overwrites the
 * buffer that a peer's stream may still be reading from the previous call.
 * Consumers of a call's Y must run on the stream passed in gpu (or
 * synchronise with it) and finish before the call after next. */
#define LLK_IPC_HANDLE_BYTES 64
typedef struct llk_peer_group llk_peer_group;

/* y_bytes: capacity of one Y buffer (>= M * N * element size of any call;
 * the group holds two). */
int llk_peer_group_create(int n_ranks, int rank, int64_t y_bytes, const llk_gpu_context *gpu, llk_peer_group **out,
                          unsigned char *ipc_handle);
/* all_handles: n_ranks * LLK_IPC_HANDLE_BYTES bytes, rank r's at r * 64. */
int llk_peer_group_connect(llk_peer_group *g, const unsigned char *all_handles);
/* The Y buffer (device) the last call wrote on this rank, and its capacity. */
int llk_peer_group_y(const llk_peer_group *g, void **y, int64_t *bytes);
/* Unmaps the peers and frees this rank's buffers.  Every rank's work on the
 * group must be finished first (e.g. synchronise the streams, then a host
 * barrier across ranks): a peer's kernel may still store into this rank's
 * buffers until its call completes.  A group is used by one host thread at
 * a time. */
void llk_peer_group_destroy(llk_peer_group *g);
/* x: device X [M, K]; this rank's weight columns as device Tensor2D pair
 * (wg_shard, wu_shard: [K, e - b]) or as packed weights (pw_shard, then
 * wg_shard / wu_shard are ignored); N = full width.  Asynchronous on
 * gpu->stream. */
int llk_swiglu_column_parallel(const Tensor2D *x, const Tensor2D *wg_shard, const Tensor2D *wu_shard,
                               const llk_packed_weights *pw_shard, int64_t N, llk_peer_group *g,
                               const llk_gpu_context *gpu);

/* ---- target probe (analogue of lib/Target/X86/TargetAVX2.cpp:33-92) ---- */

typedef struct llk_cuda_target {
  int device;
  int cc_major, cc_minor;
  int sm_count;
  int max_smem_per_block_optin; /* bytes */
  int64_t global_mem_bytes;
  int l2_bytes;
  int clock_khz;
  char name[96];
  int is_sm100a; /* 1 when the sm_100a kernels in this library can run */
} llk_cuda_target;

int llk_cuda_probe(int device, llk_cuda_target *out);

/* ---- kernel cache (device analogue of JitCache L3, JitCache.h:77-216,
 *      keyed by KernelKey, include/LLK/Runtime/KernelKey.h:45-106) -------- */

/* KernelKey field-for-field; the isa value LLK_ISA_SM100A = 16 extends
 * CpuIsa.  Value-initialise (memset 0) before filling: the cache compares
 * the whole struct, padding included, as the reference's operator== does
 * (KernelKey.h:103-105). */
enum { LLK_OP_FUSED_SWIGLU = 0, LLK_OP_MATMUL = 3, LLK_ISA_SM100A = 16 };

typedef struct llk_kernel_key {
  uint8_t operation;
  uint8_t input_type;
  uint8_t output_type;
  int64_t M_bucket;
  int64_t N;
  int64_t K;
  uint8_t weight_layout;
  uint8_t isa;
  uint8_t math_mode;
  uint16_t thread_count;
  uint64_t compiler_version;
  uint64_t schedule_version;
} llk_kernel_key;

/* The launch plan a key resolves to (what the reference caches as a
 * function pointer). */
typedef struct llk_launch_plan {
  int variant;   /* enum llk_variant */
  int block_m;   /* rows of Y per tile */
  int block_n;   /* columns of Y per tile */
  int block_k;   /* K per pipeline stage */
  int stages;    /* shared-memory pipeline depth */
  int split_k;   /* decode: K partitions; CTA-pair kernel: tail of leftover tiles, 0 = choose,
                    1/2/4 = that many column parts, -s = s K parts (2 <= s <= 8) */
  int grid;      /* CTAs launched */
  int threads;   /* threads per CTA */
  int smem_bytes;
  int sched;     /* CTA-pair kernel: 1 = static round-robin, 0 = dynamic work counter (built-in: from 12 waves of
                    tiles).  Decode kernel: 1 = one cluster of split_k CTAs per 128-column tile, partial sums
                    reduced in distributed shared memory (grid = tiles x split_k); 0 = stream-K over grid CTAs */
} llk_launch_plan;

uint64_t llk_kernel_key_hash(const llk_kernel_key *key);
int llk_plan_lookup(const llk_kernel_key *key, int64_t M, llk_launch_plan *out);
/* Installs a plan for a key (insertObjectCode, JitCache.h:116-119): a tuned
 * schedule (llk-tune) overrides the built-in choice.  A plan the kernel
 * cannot run for a call's shape is ignored at launch (the built-in plan is
 * used).  key->thread_count carries the variant and must equal
 * plan->variant. */
int llk_plan_insert(const llk_kernel_key *key, const llk_launch_plan *plan);
/* Pure lookup (lookupObjectCode, JitCache.h:113): LLK_OK with the cached
 * plan, or LLK_ERR_NOT_FOUND; builds nothing.  llk_plan_lookup is the
 * lookupOrCompile counterpart: it builds and caches the built-in plan on a
 * miss. */
int llk_plan_find(const llk_kernel_key *key, llk_launch_plan *out);
/* hits, misses, evictions of the plan cache. */
void llk_cache_stats(uint64_t *hits, uint64_t *misses, uint64_t *evictions);
void llk_cache_set_max_entries(uint64_t max_entries);
void llk_cache_clear(void);
uint64_t llk_cache_size(void);

/* Per cache level, numbered as JitCache's (1 IR, 2 optimised MLIR, 3 object
 * code, 4 packed weights): 3 is the plan cache, 4 the packed-weight cache;
 * levels 1 and 2 have no counterpart (the kernels are compiled ahead of
 * time) and report zeros / refuse with LLK_ERR_UNSUPPORTED. */
int llk_cache_level_stats(int level, uint64_t *hits, uint64_t *misses, uint64_t *evictions, uint64_t *size);
int llk_cache_level_set_max_entries(int level, uint64_t max_entries);
int llk_cache_level_clear(int level);

/* M bucket: {1}, [2,4], [5,16], [17,64], >=65 -> 0..4
 * (lib/Transforms/Common/ScheduleLoader.cpp:19-29). */
int llk_classify_m(int64_t M);

/* Library version (compiler_version in KernelKey). */
uint64_t llk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LLK_B200_H */
