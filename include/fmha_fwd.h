/*
 * fmha_fwd.h -- C ABI of the B200 (sm_100a) head-dim-64 BF16 fused multi-head
 * attention forward pass.
 *
 * This header is plain C (C99 / C++17 compatible).  BF16 tensors are passed as
 * `uint16_t*` holding the raw bf16 bit patterns; all pointers are CUDA device
 * pointers; no function allocates or frees caller memory.
 *
 * Reference interface replaced (poyenc/fmha_native):
 *   - struct FmhaFwdParams ........ src/runner/params.hpp:18-64 (same fields,
 *                                   same order, same meaning; bf16 pointers are
 *                                   uint16_t instead of __hip_bfloat16)
 *   - fmha_fwd_d64_bf16_msk0 ...... src/fused/kernel.cpp:55-63
 *   - fmha_fwd_d64_bf16_msk1 ...... src/fused/kernel.cpp:66-76
 *   - fmha_fwd_d64_bf16_msk0_varlen src/fused/kernel.cpp:80-88
 *   - fmha_fwd_d64_bf16_msk1_varlen src/fused/kernel.cpp:91-99
 * In the reference these are `__global__` kernels launched by the caller with
 * grid (nhead_q, ceil(seqlen_q/128), batch) (src/bench_fmha_fwd.cpp:174-191).
 * Here they are host functions that own the launch geometry, so the caller
 * passes the batch count explicitly (the reference passes it as gridDim.z).
 *
 * Semantics (identical to the reference):
 *   O[b,h,i,:] = softmax_j( (Q[b,h,i,:] . K[b,h/r,j,:]) / sqrt(64) ) . V[b,h/r,j,:]
 *   r = nhead_q / nhead_k (GQA/MQA).  Causal ("msk1") is bottom-right aligned:
 *   query i attends key j iff j <= i + (seqlen_k - seqlen_q).  Rows with no
 *   visible key produce O = 0 and LSE = -inf.  P is truncated to bf16 before the
 *   P.V product, as in the reference kernel; O is rounded to nearest-even bf16
 *   (the reference truncates; build with -DFMHA_O_ROUND_TRUNC for that).
 *   LSE (natural log, fp32) is written when params->lse != NULL:
 *     dense : lse[(b*nhead_q + h)*seqlen_q + i]
 *     varlen: lse[h*total_q + seqstart_q[b] + i]
 *
 * Restrictions of the TMA data path (checked, FMHA_ERR_ARG otherwise):
 *   head_dim is 64 (fixed by the entry-point name); q/k/v base pointers are
 *   16-byte aligned; every q/k/v stride is a multiple of 8 elements (16 bytes);
 *   o is 16-byte aligned with stride_o a multiple of 8 elements;
 *   nhead_q % nhead_k == 0.
 *
 * All launches are asynchronous on `stream` (NULL = legacy default stream).
 */
#ifndef FMHA_FWD_H_
#define FMHA_FWD_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st; /* cudaStream_t == struct CUstream_st* */

/* Kernel argument block.  Field order and meaning follow the reference
 * (src/runner/params.hpp:18-64).  Strides are in ELEMENTS.  `scale` is
 * pre-multiplied by log2(e): scale = log2(e)/sqrt(64). */
typedef struct FmhaFwdParams {
    const uint16_t *q, *k, *v; /* bf16 [.., seqlen, 64] with the strides below */
    uint16_t* o;               /* bf16 output, same logical layout as q        */
    float* lse;                /* optional fp32 log-sum-exp, NULL disables     */

    int seqlen_q, seqlen_k;    /* dense: lengths; varlen: max lengths          */
    int nhead_q, nhead_k;

    float scale;               /* log2(e)/sqrt(head_dim)                       */

    int stride_q, nhead_stride_q, batch_stride_q;
    int stride_k, nhead_stride_k, batch_stride_k;
    int stride_v, nhead_stride_v, batch_stride_v;
    int stride_o, nhead_stride_o, batch_stride_o;

    /* varlen: int32 prefix sums of length batch+1 (device memory); the b-th
     * sequence spans packed rows [seqstart[b], seqstart[b+1]).  Both NULL for
     * dense mode; batch_stride_* are ignored in varlen mode. */
    const int32_t* seqstart_q;
    const int32_t* seqstart_k;
} FmhaFwdParams;

/* Status codes returned by every entry point. */
enum {
    FMHA_OK = 0,
    FMHA_ERR_ARG = 1,      /* invalid argument (see restrictions above)       */
    FMHA_ERR_LAUNCH = 2,   /* CUDA launch / driver error                       */
    FMHA_ERR_TIMEOUT = 3,  /* a device-side pipeline wait exceeded its limit   */
    FMHA_ERR_DEVICE = 4,   /* no sm_100 device / unsupported device            */
    FMHA_ERR_SCRATCH = 5   /* request exceeds the allocation-free scratch      */
};

/* Dense (fixed-length batch) forward, no mask.
 * Replaces __global__ fmha_fwd_d64_bf16_msk0 (src/fused/kernel.cpp:55-63). */
int fmha_fwd_d64_bf16_msk0(const FmhaFwdParams* params, int batch,
                           struct CUstream_st* stream);

/* Dense forward, bottom-right causal mask.
 * Replaces __global__ fmha_fwd_d64_bf16_msk1 (src/fused/kernel.cpp:66-76). */
int fmha_fwd_d64_bf16_msk1(const FmhaFwdParams* params, int batch,
                           struct CUstream_st* stream);

/* Varlen (group mode) forward, no mask.  total_q / total_k are the packed row
 * counts (seqstart_q[batch], seqstart_k[batch]); they bound the TMA tensor
 * extents so no load can leave the caller's buffers.
 * Replaces __global__ fmha_fwd_d64_bf16_msk0_varlen (src/fused/kernel.cpp:80-88). */
int fmha_fwd_d64_bf16_msk0_varlen(const FmhaFwdParams* params, int batch,
                                  int total_q, int total_k,
                                  struct CUstream_st* stream);

/* Varlen forward, causal.
 * Replaces __global__ fmha_fwd_d64_bf16_msk1_varlen (src/fused/kernel.cpp:91-99). */
int fmha_fwd_d64_bf16_msk1_varlen(const FmhaFwdParams* params, int batch,
                                  int total_q, int total_k,
                                  struct CUstream_st* stream);

/* Single dispatcher over the four entries above (the host-side selection the
 * reference performs at src/bench_fmha_fwd.cpp:179-191).  Varlen is selected
 * when params->seqstart_q != NULL; total_q/total_k are ignored for dense. */
int fmha_fwd_d64_bf16(const FmhaFwdParams* params, int batch, int causal,
                      int total_q, int total_k, struct CUstream_st* stream);

/* Forward pass over an explicit list of query blocks: `tiles` is a device
 * array of `ntiles` int32 pairs (b*nhead_q + h, m) naming query block m
 * (rows [m*R, (m+1)*R), R = fmha_fwd_d64_rows_per_block()) of sequence b, head h.  Each listed block is computed exactly as
 * by the entries above; blocks not listed are left untouched.  Used to shard
 * one problem over several GPUs (every rank holds the full K/V and runs its
 * own list, no collective) and to impose a load-balanced order.  Dense or
 * varlen is selected as in fmha_fwd_d64_bf16.  No reference counterpart
 * (the reference launches every block of the grid, src/fused/kernel.cpp). */
int fmha_fwd_d64_bf16_tiles(const FmhaFwdParams* params, int batch, int causal,
                            int total_q, int total_k, const int32_t* tiles,
                            int ntiles, struct CUstream_st* stream);

/* Split-KV variant of fmha_fwd_d64_bf16_tiles for problems with too few query
 * blocks to fill the GPU (long sequences with few heads, or one rank's shard
 * of such a problem).  Every listed query block is computed as num_splits
 * independent work items over equal shares of its key range; each writes a
 * normalised fp32 partial O and its log-sum-exp into `workspace` (device
 * memory of at least fmha_fwd_d64_splitkv_workspace_bytes(ntiles, num_splits)
 * bytes, 16-byte aligned, owned by the caller), and a second kernel on the
 * same stream merges them: LSE = log sum_s exp(lse_s), O = sum_s
 * exp(lse_s - LSE) O_s.  Results equal the one-pass kernel up to fp32
 * rounding.  num_splits in [1, 64]; 1 is the plain work-list launch.  No
 * reference counterpart (the reference runs one work group per query tile
 * over the whole key range, src/fused/pipeline.hpp:286-401). */
size_t fmha_fwd_d64_splitkv_workspace_bytes(int ntiles, int num_splits);
int fmha_fwd_d64_bf16_tiles_splitkv(const FmhaFwdParams* params, int batch, int causal,
                                    int total_q, int total_k, const int32_t* tiles,
                                    int ntiles, int num_splits, void* workspace,
                                    size_t workspace_bytes, struct CUstream_st* stream);

/* Split-KV with a KV range per work item, for problems whose heaviest query
 * blocks would otherwise set the critical path (a strong-scaled shard of a
 * long causal sequence with few heads).  `items` is a device array of
 * n_items int4 records (b*nhead_q + h, m, kv_begin, kv_end), 16-byte
 * aligned, one CTA each, run in list order:
 *   kv_end <  0 : query block m over its whole key range, O/LSE written
 *                 directly (as fmha_fwd_d64_bf16_tiles);
 *   kv_end >= 0 : KV tiles [kv_begin, kv_end) (128 keys each, clipped to the
 *                 block's causal/sequence end) into partial slot `item` of
 *                 `workspace`; every run of consecutive partial items naming
 *                 the same block is merged after the launch, on the same
 *                 stream, into that block's O/LSE (LSE = log sum exp lse_s,
 *                 O = sum exp(lse_s - LSE) O_s).  A block's partial items
 *                 must be consecutive and cover its key range exactly once.
 * workspace: device memory of at least fmha_fwd_d64_items_workspace_bytes(
 * n_items) bytes, 16-byte aligned, owned by the caller.  No reference
 * counterpart (one work group per query tile over its whole key range,
 * src/fused/pipeline.hpp:286-401). */
size_t fmha_fwd_d64_items_workspace_bytes(int n_items);
int fmha_fwd_d64_bf16_items(const FmhaFwdParams* params, int batch, int causal,
                            int total_q, int total_k, const int32_t* items, int n_items,
                            void* workspace, size_t workspace_bytes,
                            struct CUstream_st* stream);

/* Allocation-free variant of fmha_fwd_d64_bf16_tiles.  No counterpart in the
 * reference.  Meant for callers that may not allocate device memory: code
 * running where cudaMalloc is refused or would stall the device (inside a
 * stream capture, a serving loop that must never synchronise) or a plug-in
 * whose host framework owns all allocations.  The regular entries allocate a
 * 4-byte error word per device on first use; this one allocates nothing and
 * keeps its scratch -- the error word and a copy of the work list -- in a
 * fixed 128 KB array inside the library (held by every GPU that loads it).
 *   host_tiles : HOST array of ntiles int32 pairs (b*nhead_q + h, m), as for
 *                fmha_fwd_d64_bf16_tiles.  Every entry is checked on the host
 *                first (FMHA_ERR_ARG, nothing queued, if one names a (batch,
 *                head) or query block outside the problem).  The list is then
 *                copied with cudaMemcpyAsync on `stream`.  From pageable
 *                memory the copy is staged before the call returns, so the
 *                array may be reused at once; from pinned (page-locked)
 *                memory the GPU reads it when the copy executes, so it must
 *                stay unchanged until the stream has executed the call.
 *   ntiles     : at most 16384, else FMHA_ERR_SCRATCH and nothing is launched.
 * The first call on a device resolves the scratch address for that device
 * (make it before any stream capture begins).  All calls share the one array
 * and each call overwrites it: calls whose executions overlap on the GPU race
 * and must be serialised (e.g. one stream).  Read device timeouts with
 * fmha_fwd_d64_noalloc_status, which clears the error word it reports. */
int fmha_fwd_d64_bf16_tiles_noalloc(const FmhaFwdParams* params, int batch, int causal,
                                    int total_q, int total_k, const int32_t* host_tiles,
                                    int ntiles, struct CUstream_st* stream);

/* Synchronizes `stream` and reports FMHA_ERR_TIMEOUT if a pipeline wait of an
 * allocation-free call since the last report expired (FMHA_OK otherwise);
 * the error word is cleared when it is reported.  No counterpart in the
 * reference. */
int fmha_fwd_d64_noalloc_status(struct CUstream_st* stream);

/* Synchronizes `stream`, then reads and clears the device error word written
 * by bounded pipeline waits on the current device.  Returns FMHA_OK or
 * FMHA_ERR_TIMEOUT (or FMHA_ERR_LAUNCH if the synchronization failed).
 * No reference counterpart (the reference kernel has no error reporting). */
int fmha_fwd_d64_status(struct CUstream_st* stream);

/* Sets the time limit (nanoseconds) of every device-side pipeline wait for
 * subsequent launches on all devices; 0 restores the default (2 s).
 * No reference counterpart. */
void fmha_fwd_d64_set_wait_limit_ns(unsigned long long limit_ns);

/* Releases the per-device launcher context (error word).  No reference
 * counterpart. */
void fmha_fwd_d64_release(void);

/* Human-readable text for a status code. */
const char* fmha_fwd_d64_error_string(int status);

/* Query rows per work-list entry of the built kernel (128: one 128-row query
 * tile per work item).  No reference counterpart. */
int fmha_fwd_d64_rows_per_block(void);

/* Tile geometry of the B200 kernel (informational; callers need not compute
 * launch geometry).  128 query rows per tile, one tile per CTA, two CTAs per
 * SM, 128 keys per KV tile. */
#define FMHA_B200_BLOCK_M 128
#define FMHA_B200_ROWS_PER_BLOCK 128 /* query rows per work-list entry (see fmha_fwd_d64_rows_per_block) */
#define FMHA_B200_BLOCK_N 128
#define FMHA_B200_HEAD_DIM 64

#ifdef __cplusplus
}
#endif

#endif /* FMHA_FWD_H_ */
