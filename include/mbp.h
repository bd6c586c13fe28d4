/*
 * mbp.h -- C ABI of the B200 (sm_100a) small-M projection library (libmbp.so).
 *
 * The library computes out[M, N] = x[M, K] . W[N, K]^T for small token counts M from weights stored in a
 * lossless 12-bit BF16 format, plus the FP32 router as a BF16 hi/lo pair.  Plain pointers and sizes only: all
 * pointers are DEVICE pointers unless stated, every call is asynchronous on the given CUDA stream and returns
 * MBP_OK (0) or a negative status (the reference's convention, submission.py sm_launch S:46<494-552>).
 *
 * Each entry point names the reference interface it replaces (reference = NathenFernandes/muse-bf16-proj,
 * file submission.py, "S:<line>"; "S:46<a-b>" = lines a-b of the CUDA text stored compressed on line 46).
 */
#ifndef MBP_H
#define MBP_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (S:46<494-552>: -1 threads, -2 N%RB, -3 K split, -5 m range, -6 smem, -8 launch,
 *      -9 cluster, -99 unknown instance, -100 tensor-map encode) ---- */
#define MBP_OK 0
#define MBP_ERR_ARG (-1)      /* null pointer or bad enum */
#define MBP_ERR_SHAPE (-2)    /* n % 16, k % 64, n_out > n, or chunk count >= 32767 */
#define MBP_ERR_SPLIT (-3)    /* impossible geometry */
#define MBP_ERR_ALIGN (-4)    /* pointer not 16-byte aligned */
#define MBP_ERR_M (-5)        /* token count out of range */
#define MBP_ERR_SMEM (-6)     /* shared memory request above the device limit */
#define MBP_ERR_LAUNCH (-8)   /* cudaLaunchKernelEx failed (cudaGetLastError is left set) */
#define MBP_ERR_CLUSTER (-9)  /* cluster shape not schedulable */
#define MBP_ERR_DEVICE (-10)  /* device is not sm_100 */
#define MBP_ERR_CAP (-11)     /* caller buffer too small */
#define MBP_ERR_TMAP (-100)   /* cuTensorMapEncodeTiled failed */
#define MBP_ERR_SCRATCH_LIMIT (-12) /* matrix too tall for the fixed scratch of mbp_pack_c12_noalloc */

/* device status word codes (written by bounded waits instead of trapping; read with mbp_status) */
#define MBP_DEV_TIMEOUT_FULL 1   /* consumer gave up waiting for a stage's bytes */
#define MBP_DEV_TIMEOUT_EMPTY 2  /* producer gave up waiting for a stage to drain */
#define MBP_DEV_TIMEOUT_MMA 3    /* tensor-core completion did not arrive */
#define MBP_DEV_TIMEOUT_PEER 4   /* a peer rank's barrier flag did not arrive */

/* ---- weight formats ---- */
#define MBP_UNIT_ROWS 16
#define MBP_UNIT_COLS 64
#define MBP_C12_UNIT_BYTES 1536 /* 1024 weights x 12 bits */
#define MBP_RAW_UNIT_BYTES 2048 /* 1024 weights x 16 bits */

#define MBP_BASE_MATRIX 0 /* one exponent base per matrix: byte-identical to the reference (S:104-125) */
#define MBP_BASE_TILE 1   /* one exponent base per 16-row tile */

/* A 12-bit packed matrix W[n, k] in device memory (layout: S:82-125 units, generalised escape list).
 *   units   [n/16][k/64][1536] bytes, row-tile major
 *   bases   [n/16]  exponent base (7 high exponent bits) of each 16-row tile
 *   esc_off [(n/16)*(k/64) + 1] int32: escapes of unit u are esc[esc_off[u] .. esc_off[u+1])
 *   esc     [n_esc] uint32 entries  chunk << 17 | lane << 12 | value << 7 | xor7  (NULL when n_esc == 0) */
typedef struct mbp_c12 {
  const uint8_t* units;
  const uint8_t* bases;
  const int32_t* esc_off;
  const uint32_t* esc;
  int32_t n;
  int32_t k;
  int64_t n_esc;
} mbp_c12;

/* An FP32 matrix stored as a BF16 hi/lo pair (S:876-879), uncompressed units (S:98-101):
 *   units [n/16][k/64][2][2048] bytes: the hi unit then the lo unit of each 16x64 block. */
typedef struct mbp_hilo {
  const uint8_t* units;
  int32_t n;
  int32_t k;
} mbp_hilo;

/* Launch geometry of the weight-streaming GEMV.  Zero-initialise and call mbp_gemv_plan, or fill by hand. */
typedef struct mbp_gemv_geom {
  int32_t rb;      /* 16-row tiles per CTA */
  int32_t rtw;     /* 16-row tiles per consumer warp (1 or 2) */
  int32_t split;   /* CTAs splitting K = cluster size (1..16) */
  int32_t wki;     /* consumer warps splitting a CTA's K range */
  int32_t kci;     /* 64-column chunks per consumer warp per pipeline stage */
  int32_t stages;  /* pipeline depth */
  int32_t nblk;    /* CTAs along the rows, tiles split evenly (at most rb each); 0 = ceil(n_out/16 / rb) */
} mbp_gemv_geom;

/* ---- library / device ---- */
int mbp_version(void);
/* 0 when `device` is an sm_100 part this library was built for. */
int mbp_device_check(int device);
/* Reads (and with clear != 0 resets) the device status word after the stream has been synchronised. */
int mbp_status(int* status, int clear);
/* Limit, in nanoseconds, of every bounded device wait (pipeline stages, tensor-core completion, peer words and
 * flags) in the kernels launched from now on, process-wide; 0 restores the default of 1 s.  Returns the previous
 * limit.  A wait that runs out records its MBP_DEV_TIMEOUT_* code in the status word and the kernel returns
 * instead of trapping (replaces the reference's __trap() after a 20 ms spin, S:46<105-111>).  A launch captured
 * in a CUDA graph keeps the limit that was in force at capture. */
unsigned long long mbp_set_wait_limit(unsigned long long ns);

/* ---- GPU packer (replaces the host-side torch packer sm_units/sm_c12_bytes/sm_stream, S:82-227) ----
 * Two phases, because the escape count is known only after the first:
 *   1. mbp_pack_c12 writes units, bases and esc_off (esc_off[(n/16)*(k/64)] = total escape count);
 *   2. after reading that total, the caller allocates esc and calls mbp_pack_c12_escapes.
 * `workspace` must hold mbp_pack_c12_workspace(n, k) bytes. w is BF16 row-major [n, k], 16-byte aligned. */
size_t mbp_pack_c12_workspace(int n, int k);
int mbp_pack_c12(const uint16_t* w, int n, int k, int base_mode, uint8_t* units, uint8_t* bases, int32_t* esc_off,
                 void* workspace, size_t workspace_bytes, cudaStream_t stream);
/* Allocation-free phase 1 of the packer.  No counterpart in the reference.  For callers that cannot allocate
 * device memory themselves: a loader handed only preallocated weight and output buffers by a host framework
 * that owns all device memory, or a caller that must not trigger cudaMalloc's implicit device-wide
 * synchronisation while other streams run.  Same arguments and results as mbp_pack_c12 minus the workspace:
 * the per-tile histograms live in a fixed 512 KiB device array inside the library (held by every GPU that
 * loads the library until the process exits), which limits n to 16384 rows (MBP_ERR_SCRATCH_LIMIT beyond).
 * Calls no cudaMalloc/cudaFree.  Its first call on a device looks up the array's device address, so make that
 * first call before any stream capture.  All calls share the array: calls that overlap on the GPU (other
 * streams, other threads) race on it; serialise them. */
int mbp_pack_c12_noalloc(const uint16_t* w, int n, int k, int base_mode, uint8_t* units, uint8_t* bases,
                         int32_t* esc_off, cudaStream_t stream);
int mbp_pack_c12_escapes(const uint16_t* w, int n, int k, const uint8_t* bases, const int32_t* esc_off,
                         uint32_t* esc, cudaStream_t stream);
/* Exact inverse (verification on the device, like the reference's sm_c12_unpack check S:168-170). */
int mbp_unpack_c12(const mbp_c12* w, uint16_t* w_out, cudaStream_t stream);

/* FP32 [n, k] -> hi/lo units (S:876-879 split + S:98-101 layout). */
int mbp_pack_hilo(const float* w, int n, int k, uint8_t* units, cudaStream_t stream);

/* ---- weight-streaming GEMV, M <= 32 per token block (replaces sm_launch S:48-53 / S:46<555-561> and its
 * clones m32_launch S:418-423, the mw launcher S:2398, the smallm2/smtrace/v18 GEMVs) ----
 * out[m, n_out] = x[m, k] . W[0:n_out, :]^T, FP32 accumulation.  x BF16 row-major [m, k] (16-byte aligned);
 * out BF16 (mbp_gemv_c12) or FP32 (mbp_gemv_c12_f32) row-major with leading dimension ldo (elements).
 * n_out <= n, n_out % 16 == 0 (the reference's unpooler uses the first 1024 rows at M <= 8, S:272-273).
 * m >= 1; m > 32 runs 32-token blocks.  geom may be NULL (planned internally, for the matrix's escape count and
 * the output type).  mbp_gemv_plan plans for a matrix with dense escapes and BF16 output (valid for every
 * matrix); mbp_gemv_plan_ex takes MBP_PLAN_* flags and returns exactly the geometry a NULL geom would use. */
#define MBP_PLAN_ESCAPES 1       /* the matrix has escapes (n_esc > 0): consumer warps reserve escape masks */
#define MBP_PLAN_F32_OUT 2       /* FP32 output (mbp_gemv_c12_f32) */
#define MBP_PLAN_DENSE_ESCAPES 4 /* at least one escape per 1000 weights (n_esc * 1000 >= n * k) */
int mbp_gemv_plan(int n_out, int k, int m, mbp_gemv_geom* geom);
int mbp_gemv_plan_ex(int n_out, int k, int m, int flags, mbp_gemv_geom* geom);
int mbp_gemv_c12(const mbp_c12* w, const uint16_t* x, int m, int n_out, uint16_t* out, int ldo,
                 const mbp_gemv_geom* geom, cudaStream_t stream);
int mbp_gemv_c12_f32(const mbp_c12* w, const uint16_t* x, int m, int n_out, float* out, int ldo,
                     const mbp_gemv_geom* geom, cudaStream_t stream);

/* ---- verify-path GEMM on the tcgen05 tensor cores (replaces the dense BF16 verify GEMMs ss_gemm S:783,
 * q_kernel S:979 / qb_kernel S:4576, ol_projection S:1547, projection S:2985, and the out-of-scope cuBLASLt routes
 * S:2309-2376): out[m, n_out] = x . W[0:n_out]^T, FP32 accumulation in TMEM, any m >= 1 (tiles of up to 256
 * tokens; intended for m > 32).  The weights stay packed in HBM; decoded tiles go to TMEM as the MMA's A
 * operand.  Short-K shapes split the tokens into tiles, few-tile shapes split K over a thread-block cluster
 * (reduced in distributed shared memory, a fixed order: repeated calls give identical bits). ---- */
int mbp_gemm_c12(const mbp_c12* w, const uint16_t* x, int m, int n_out, uint16_t* out, int ldo,
                 cudaStream_t stream);
int mbp_gemm_c12_f32(const mbp_c12* w, const uint16_t* x, int m, int n_out, float* out, int ldo,
                     cudaStream_t stream);

/* ---- tensor-parallel helpers (no counterpart in the reference, which is single-GPU) ----
 * Column-parallel: each rank computes a [m, ns] shard of out; an all-gather into one buffer yields [P][m][ns];
 * mbp_tp_assemble_columns writes the row-major [m][P*ns] output (ns % 8 == 0).
 * Row-parallel: each rank computes FP32 partial sums of the full output from its K slice; after the NCCL sum,
 * mbp_f32_to_bf16 rounds them to the BF16 output (n % 4 == 0). */
int mbp_tp_assemble_columns(const uint16_t* gathered, uint16_t* out, int P, int m, int ns, cudaStream_t stream);
int mbp_f32_to_bf16(const float* in, uint16_t* out, long long n, cudaStream_t stream);

/* Peer-store exchange on one node (NVLink peers mapped through CUDA IPC; plain loads and stores, no multicast).
 * mbp_ipc_alloc: zeroed device buffer + its 64-byte IPC handle; mbp_ipc_open maps a peer's buffer into this
 * process (mbp_ipc_close unmaps, mbp_ipc_free releases an own buffer).
 * mbp_gemv_c12_multi: the GEMV of mbp_gemv_c12(_f32) storing the same result into `nout` (<= 8) outputs with
 * one leading dimension, outs[0] local, the others peers' buffers; x rows are ldx elements apart (ldx >= k,
 * ldx % 8 == 0), so a rank reads its column slice of a wider x in place.  out_kind:
 *   MBP_OUT_BF16 / MBP_OUT_F32  plain [m][ldo] outputs;
 *   MBP_OUT_TAGGED_BF16X2       64-bit words [m][ldo] (ldo >= n_out/2): word (t, 8*tile + g) = bf16 rows
 *                               16*tile + g (low half) and 16*tile + g + 8 (high half), tag in the upper 32 bits;
 *   MBP_OUT_TAGGED_F32          64-bit words [m][ldo] (ldo >= n_out): word (t, row) = f32 bits | tag << 32.
 * The tagged kinds need `epoch` (the plain kinds ignore it and parity_stride): this call's epoch is
 * (*epoch + 1), the tag, and every output pointer moves by parity_stride bytes when it is odd (the exchange
 * buffer mbp_tp_finish with the same counter reads).  A tagged word and its tag travel in one 64-bit store, so
 * no fence is needed between ranks.
 * mbp_tp_finish: counter = this rank's MBP_TP_COUNTER_SLOTS epoch slots (zero-initialised device memory, shared
 * by every exchange of one group); advances the epoch and, by mode:
 *   MBP_TP_BARRIER      flags[r] = rank r's flag array (8 ints, zero-initialised): announces the epoch to every
 *                       rank after a system fence that orders this rank's earlier stores (stream order) before
 *                       it, and waits (bounded, MBP_DEV_TIMEOUT_PEER) until every rank announced it;
 *   MBP_TP_GATHER_BF16  waits (bounded) until every word of buf's parity half [m][n/2] carries the epoch's tag
 *                       (written by the P ranks' MBP_OUT_TAGGED_BF16X2 GEMVs) and writes out[m][n] bf16;
 *   MBP_TP_SUM_F32      waits likewise on P slots [P][m][n] of MBP_OUT_TAGGED_F32 words and writes
 *                       out[t][i] = bf16(sum_r slot_r[t][i]) in rank order (identical on every rank).
 * The tagged modes launch as programmatic dependents of the GEMV before them, so they poll while it drains.
 * Every rank of a group must make the same sequence of calls.  Graph-replayable. */
#define MBP_TP_COUNTER_SLOTS 64
#define MBP_TP_BARRIER 0
#define MBP_TP_GATHER_BF16 1
#define MBP_TP_SUM_F32 2
#define MBP_TP_RSAG 3
#define MBP_OUT_BF16 0
#define MBP_OUT_F32 1
#define MBP_OUT_TAGGED_BF16X2 2
#define MBP_OUT_TAGGED_F32 3
int mbp_ipc_alloc(size_t bytes, void** ptr, void* handle64);
int mbp_ipc_open(const void* handle64, void** ptr);
int mbp_ipc_close(void* ptr);
int mbp_ipc_free(void* ptr);
/* mbp_gemm_c12_multi: the tcgen05 GEMM (any m) storing its result as MBP_OUT_TAGGED_BF16X2 words (column-parallel
 * gather; receive: mbp_tp_finish MBP_TP_GATHER_BF16) or MBP_OUT_TAGGED_F32 words (row-parallel partials; receive:
 * MBP_TP_SUM_F32) into `nout` (<= 8) exchange buffers, same layout, epoch and parity rules as mbp_gemv_c12_multi.
 * The exchange of the verify-size calls, in place of an NCCL collective and its assembly / rounding kernel. */
int mbp_gemm_c12_multi(const mbp_c12* w, const uint16_t* x, int m, int n_out, void* const* outs, int nout, int ldo,
                       int out_kind, const int* epoch, long long parity_stride, cudaStream_t stream);
int mbp_gemv_c12_multi(const mbp_c12* w, const uint16_t* x, int ldx, int m, int n_out, void* const* outs, int nout,
                       int ldo, int out_kind, const int* epoch, long long parity_stride, const mbp_gemv_geom* geom,
                       cudaStream_t stream);
int mbp_tp_finish(int* const* flags, int rank, int P, int* counter, const void* buf, long long parity_stride,
                  int mode, int m, int n, void* out, cudaStream_t stream);

/* Tensor-parallel projection in ONE kernel per call: the GEMV of this rank's shard stores its results as
 * epoch-tagged words into every rank's exchange buffer (plain NVLink stores), then each CTA waits (bounded,
 * MBP_DEV_TIMEOUT_PEER) for the same tiles from the other ranks in its own buffer and writes them into `out`
 * [m][n] (BF16): gathered columns (MBP_TP_GATHER_BF16, column-parallel: w holds rows [rank*n/P, (rank+1)*n/P))
 * or the rank-order sum of the FP32 partials (MBP_TP_SUM_F32, row-parallel: w holds n rows and x's columns
 * [rank*k, (rank+1)*k) for w's k, read in place through ldx: every rank sends its whole partial to every rank),
 * or the same sum as a reduce-scatter + gather (MBP_TP_RSAG: the tiles of CTA (x, z) belong to rank
 * (x + z) % P, which alone receives their partials, adds them in rank order and sends the BF16 result as bf16x2
 * words into every rank's gather region at byte P*32*n*8 of each buffer half, which must hold [32][n/2] words
 * more: (P-1)/P x 12 m n bytes leave each rank instead of (P-1) x 8 m n).  The grid's last CTA advances the epoch (counter:
 * MBP_TP_COUNTER_SLOTS slots + one ticket int, zero-initialised).  Exchange buffers: two parity halves of
 * m*n/2 (gather) or P*m*n (sum) 64-bit words each.  Every rank makes the same sequence of calls; each rank's
 * grid must fit one wave (the planner's geometries do); graph-replayable. */
typedef struct {
  void* bufs[8];            /* rank r's exchange buffer as mapped in this process, r < P */
  long long parity_stride;  /* bytes between a buffer's two parity halves (multiple of 16) */
  int* counter;             /* this rank's epoch slots and ticket */
  int rank, P;
  int mode;                 /* MBP_TP_GATHER_BF16 or MBP_TP_SUM_F32 */
  int n;                    /* output columns of the whole projection */
} mbp_tp_exchange;
int mbp_gemv_c12_tp(const mbp_c12* w, const uint16_t* x, int ldx, int m, const mbp_tp_exchange* ex, uint16_t* out,
                    const mbp_gemv_geom* geom, cudaStream_t stream);

/* ---- FP32 router through the hi/lo pair (replaces rr_launch / rr_scalar / rr_small S:856-861, routertail
 * S:5424, rwdl S:5377): out_f32[m, n] = x . hi^T + x . lo^T, FP32 accumulation. ---- */
int mbp_router_hilo(const mbp_hilo* w, const uint16_t* x, int m, float* out, int ldo, const mbp_gemv_geom* geom,
                    cudaStream_t stream);
/* The same product on the tcgen05 tensor cores (replaces the wide-router family rwdl_128 / rwdl_256, S:5377):
 * A = the hi and lo units in TMEM, two MMAs per K step into one FP32 accumulator, the K range split over a
 * thread-block cluster (<= 16) reduced in a fixed order through distributed shared memory.  bn = token tile
 * (multiple of 16, <= 128; 0 = default), split = cluster size (<= 16, and >= k / 2048 so that no CTA accumulates
 * more than 2048 columns on the tensor pipe, which keeps the 1e-5 accuracy; 0 = choose); k <= MBP_ROUTER_TC_MAX_K.
 * mbp_router_hilo takes this path when geom is NULL, m >= MBP_ROUTER_TC_MIN_M and k <= MBP_ROUTER_TC_MAX_K. ---- */
#define MBP_ROUTER_TC_MIN_M 257 /* measured: the GEMV is faster up to 256 tokens, this path from 384 */
#define MBP_ROUTER_TC_MAX_K 32768
int mbp_router_hilo_tc(const mbp_hilo* w, const uint16_t* x, int m, float* out, int ldo, int bn, int split,
                       cudaStream_t stream);

/* ---- Router consumer (no counterpart in the reference, which stops at the logits): the k largest of each
 * token's e logits (rows ld floats apart; e <= 1024, k <= min(e, 32)), ids[t][j] in descending logit order (equal
 * logits: lower index first; NaN below every number), weights[t][j] = softmax over the k selected logits
 * (renorm = 1) or the full softmax over all e, taken at the selected ones (renorm = 0).  Launched as a
 * programmatic dependent of the kernel before it (the router GEMV), whose completion it waits for. ---- */
int mbp_router_topk(const float* logits, int m, int e, int ld, int k, int renorm, float* weights, int32_t* ids,
                    cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MBP_H */
