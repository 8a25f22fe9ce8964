// fmha_fwd_kernel.cu -- B200 (sm_100a) head-dim-64 BF16 fused attention
// forward, and the C-ABI launchers declared in include/fmha_fwd.h.
//
// One CTA owns one 128-row query tile of one (batch, head) and walks the
// key/value sequence in 128-key tiles; two CTAs share each SM, each with its
// own pipeline.  The CTA is warp specialised:
//
//   warps 0-3  softmax          : one query row per thread (TMEM lane = row)
//   warp  4    TMA producer     : Q once, then K_j / V_j into a 4-slot ring
//   warp  5    MMA issuer       : one elected lane issues every tcgen05.mma;
//                                 the warp also owns the TMEM allocation
//   warps 6-7  idle             : complete the control warpgroup for setmaxnreg
//
// Tensor memory (256 columns x 128 lanes per CTA; two CTAs fill the SM):
//   [  0,128) S = Q K^T (fp32)
//   [128,192) O accumulator (fp32)
//   [192,256) P (bf16x2)
//
// Per KV tile j the schedule is
//   MMA : S = Q K_j^T -> commit(s_full)
//   SM  : S -> registers -> arrive(s_free) -> mask, row max, (lazy) rescale
//         of O -> P = exp2(S*scale - m*scale) -> wait(pv_done of j-1) ->
//         bf16 P into TMEM -> arrive(p_full)
//   MMA : S = Q K_{j+1}^T as soon as s_free arrives, then O += P V_j ->
//         commit(pv_done)
// tcgen05 MMAs issued by one thread execute in order, so pv_done(j-1) also
// proves every earlier MMA finished, which is what makes the softmax-side O
// rescale race free.
//
// The exp2 reference m: the first pass takes the exact row max of the first
// KV tile and keeps it for every later tile (no row max there); a tile whose
// row sum of P exceeds 2^40 means the reference was outgrown, and the CTA
// then runs a second, exact pass (running max, lazy rescale) over the same
// tiles, continuing every barrier phase on a flat step index.
//
// CTAs start in work order (heaviest query tiles first inside L2-sized head
// groups), so the hardware block scheduler balances the load dynamically.  A
// persistent variant (two resident CTAs per SM looping over the tiles, Q
// double-buffered, the next tile's first QK^T issued before the current
// tile's last PV) measured 4-8 % slower on every north-star shape: the
// neighbouring CTA already hides one CTA's start and finish.
//
// Reference semantics followed (poyenc/fmha_native):
//   grid decode + causal heavy-first order ... src/fused/kernel.cpp:55-99
//   varlen offsets, causal KV end ........... src/fused/pipeline.hpp:116-193
//   degenerate tile (no key) -> O=0, LSE=-inf src/fused/pipeline.hpp:207-222
//   boundary / causal masking ............... src/fused/op_softmax.hpp:73-131
//   exp2 softmax with log2e-folded scale .... src/fused/op_softmax.hpp:148-255
//   P truncated to bf16 before P.V .......... src/fused/op_gemm.hpp:272-273
//   O * (1/l), LSE .......................... src/fused/op_epilog.hpp:50-155
//     (O is rounded to nearest-even bf16 by default, halving the error
//      against the fp32 oracle; -DFMHA_O_ROUND_TRUNC restores the
//      reference kernel's truncation, op_epilog.hpp:103-124)
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <vector>

#include "../../include/fmha_fwd.h"
#include "sm100_ptx.cuh"

using namespace fmha_sm100;

namespace {

constexpr int kBlockM = 128;            // rows per query tile
constexpr int kBlockN = 128;            // keys per KV tile
constexpr int kHeadDim = 64;
// One CTA = one 128-row query tile (128 query rows, 256 threads, 256 TMEM
// columns, ~80 KB shared memory); two CTAs run per SM, each with its own
// pipeline, fully independent of its neighbour.  The per-tile arrays and
// loops below run over that one tile.
constexpr int kTilesPerCta = 1;
constexpr int kRowsPerCta = kBlockM * kTilesPerCta;
constexpr int kCtasPerSm = 2;
constexpr int kStages = 4;              // K/V ring slots (K_j, V_j alternate)
constexpr int kTileBytes = kBlockM * kHeadDim * 2;  // 16 KB (Q, K or V tile)
constexpr int kWarpsPerTile = 4;   // softmax warps per query tile: one thread per row
constexpr int kSoftmaxWarps = kWarpsPerTile * kTilesPerCta;
constexpr int kThreads = 32 * kSoftmaxWarps + 128;  // softmax group + control group
// Register split (setmaxnreg): the CTA launches with kThreads x kLaunchRegs
// registers; the softmax group takes kRegsSoftmax, the producer/MMA group
// kRegsControl: 128 * (192 + 64) <= 256 * 128.
constexpr int kRegsSoftmax = 192;
constexpr int kRegsControl = 64;
constexpr int kLaunchRegs = 128;
static_assert(32 * kSoftmaxWarps * kRegsSoftmax + 128 * kRegsControl <= kThreads * kLaunchRegs,
              "setmaxnreg split exceeds the launch register pool");
constexpr int kWarpLoad = kSoftmaxWarps;
constexpr int kWarpMma = kSoftmaxWarps + 1;
constexpr uint32_t kTmemCols = 256 * kTilesPerCta;
__host__ __device__ constexpr uint32_t col_s(int i) { return i * 128u; }        // S_i (fp32)
__host__ __device__ constexpr uint32_t col_o(int i) { return 128u * kTilesPerCta + i * 64u; }  // O_i
__host__ __device__ constexpr uint32_t col_p(int i) {  // P_i (bf16x2)
    return 192u * kTilesPerCta + i * 64u;
}
// Lazy rescale threshold in log2 units: the running max is only moved when
// it grows by more than this, bounding un-normalised P by 2^8.
constexpr float kRescaleThreshold = 8.0f;
// P is truncated to bf16 before P V, which lowers it by 0.28 % on average
// (half a bf16 step, 2^-8 times the mean of 1/mantissa, 1/ln 4).  The
// exponent is raised by log2(1 + 0.002818) so the truncation is centred;
// l and the LSE see the same factor, which the LSE removes again.  Without
// it a row dominated by one key (whose P the lazy reference leaves anywhere
// in [1, 2^8)) loses up to 0.78 % of its output.
constexpr float kPLog2Bias = 0.0040614f;
// Pairs (of every 16) whose exp2 runs as a polynomial on the FMA/ALU pipes
// instead of MUFU (unmasked tiles only).
#ifndef FMHA_EXP_POLY_PAIRS
#define FMHA_EXP_POLY_PAIRS 4
#endif
constexpr int kExpPolyPairs = FMHA_EXP_POLY_PAIRS;

// Error codes written to the device error word.
constexpr int kErrTimeoutLoad = 0x101;
constexpr int kErrTimeoutMma = 0x102;
constexpr int kErrTimeoutSoftmax = 0x103;

// Trace builds (-DFMHA_TRACE, libfmha_b200_trace.so): clock64 stamps of the
// pipeline events of pass 0 for kTraceCtas consecutive CTAs, kTraceSteps KV
// steps each, kTraceSlots events per step (the slot map is in
// fmha_native_b200/trace.py).  In the product library the stamps compile
// to nothing.
#ifdef FMHA_TRACE
constexpr int kTraceCtas = 64;
constexpr int kTraceSteps = 64;
constexpr int kTraceSlots = 16;
__device__ int g_trace_cta0 = 0;
__device__ unsigned long long g_trace[kTraceCtas * kTraceSteps * kTraceSlots];
__device__ __forceinline__ unsigned smid() {
    unsigned r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}
// Row of this CTA in the trace buffer (-1: not traced); read once per CTA.
#define FMHA_TRACE_INIT const int trace_row_ = (int)blockIdx.x - g_trace_cta0
#define FMHA_TRACE_AT(slot, j, val)                                                    \
    do {                                                                               \
        if (trace_row_ >= 0 && trace_row_ < kTraceCtas && (j) >= 0 && (j) < kTraceSteps) \
            g_trace[(trace_row_ * kTraceSteps + (j)) * kTraceSlots + (slot)] = (val);   \
    } while (0)
#else
#define FMHA_TRACE_INIT \
    do {                \
    } while (0)
#define FMHA_TRACE_AT(slot, j, val) \
    do {                            \
    } while (0)
#endif
#define FMHA_TRACE_CLOCK(slot, j) FMHA_TRACE_AT(slot, j, clock64())

struct KernelArgs {
    CUtensorMap tm_q;
    CUtensorMap tm_k;
    CUtensorMap tm_v;
    uint16_t* o;
    float* lse;
    const int32_t* seqstart_q;
    const int32_t* seqstart_k;
    const int32_t* seq_order;  // varlen launch order: slot -> sequence, longest first (or null)
    const int2* block_map;     // compact varlen launch: CTA / nhead_q -> (sequence, query block)
    long long stride_o, nhead_stride_o, batch_stride_o;
    int seqlen_q, seqlen_k;
    int nhead_q, nhead_k;
    int total_q;               // varlen: LSE head stride
    float scale;
    int* err_word;
    unsigned long long wait_limit_ns;
    int stall_inject;          // test hook: producer withholds the first V tile
    const int32_t* tiles;      // optional work list of (b*nhead_q+h, query block)
    int m_blocks;              // query blocks per (batch, head) in a full launch
    int head_group;            // (batch, head) pairs per L2 group of the launch order
    int num_hb;                // batch * nhead_q
    int num_splits;            // split-KV: work item x = (tiles[x / num_splits], KV range x % num_splits)
    const int32_t* items;      // optional work items (b*nhead_q+h, query block, kv_begin, kv_end)
    float* part_o;             // split-KV partial O (fp32, normalised) [item][128][64]
    float* part_lse;           // split-KV partial LSE (natural log) [item][128]
};

struct alignas(1024) SharedStorage {
    uint8_t q[kTilesPerCta][kTileBytes];
    uint8_t kv[kStages][kTileBytes];
    uint64_t bar_q[kTilesPerCta];
    uint64_t bar_full[kStages];
    uint64_t bar_empty[kStages];
    uint64_t bar_s[kTilesPerCta];      // S_i written (MMA commit)
    uint64_t bar_sfree[kTilesPerCta];  // S_i read into registers (128 arrivals)
    uint64_t bar_p[kTilesPerCta];      // P_i written, O_i rescaled (128 arrivals)
    uint64_t bar_pv[kTilesPerCta];     // O_i += P_i V done (MMA commit)
    uint64_t bar_o[kTilesPerCta];
    uint64_t bar_drain;
    uint64_t bar_dec;                  // softmax's verdict on the first pass (128 arrivals)
    uint32_t tmem_base;
    int abort_flag;
    int rerun;                         // a row's scores outgrew the fixed reference: exact pass
};

// Bounded wait on an mbarrier phase.  Returns false if the CTA-wide abort
// flag is raised or the time limit expires (then it raises the flag and
// records `code` in the device error word).
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                        const KernelArgs& a, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > a.wait_limit_ns) {
                *abort_flag = 1;
                atomicCAS(a.err_word, 0, code);
                return false;
            }
        }
    }
}

// Bounded wait used only while tearing down after an abort: ignores the
// abort flag, gives up silently after the time limit.
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity, const KernelArgs& a) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > a.wait_limit_ns) return;
    }
}

struct TileWork {
    int n_kv[kTilesPerCta];     // KV tiles each query tile walks (from j0)
    int j0;                     // first KV tile (split-KV ranges start past 0)
    int row0;                   // first query row of the CTA (sequence-local)
    int seqlen_q, seqlen_k;
    int off_q, off_k;           // varlen packed-row offsets
    int b, h, kvh;
    bool partial;               // split-KV item: partial O/LSE into the workspace
};

template <bool kCausal, bool kVarlen>
__device__ __forceinline__ bool decode_work(const KernelArgs& a, TileWork& w) {
    int hb, mblk;
    int split = 0;
    int kv_begin = 0, kv_end = -1;  // work items: explicit KV-tile range (end < 0: all)
    if (a.items != nullptr) {
        const int4 it = reinterpret_cast<const int4*>(a.items)[blockIdx.x];
        hb = it.x;
        mblk = it.y;
        kv_begin = it.z;
        kv_end = it.w;
        if (kv_end >= 0 && (kv_begin < 0 || kv_begin > kv_end)) return false;
    } else if (a.tiles != nullptr) {
        // Caller-supplied work list: (batch*nhead_q + head, query block); in
        // split-KV mode every entry expands into num_splits KV ranges.
        const int x = a.num_splits > 1 ? (int)blockIdx.x / a.num_splits : (int)blockIdx.x;
        if (a.num_splits > 1) split = (int)blockIdx.x % a.num_splits;
        hb = a.tiles[2 * x];
        mblk = a.tiles[2 * x + 1];
    } else if (kVarlen && a.block_map != nullptr) {
        // Compact varlen launch: nhead_q consecutive CTAs per query block,
        // blocks in the order of the map (longest sequence first).
        const int2 e = a.block_map[(int)blockIdx.x / a.nhead_q];
        if (e.x < 0) return false;  // past the last block
        hb = e.x * a.nhead_q + (int)blockIdx.x % a.nhead_q;
        mblk = e.y;
    } else {
        // Launch order: (batch, head) pairs in groups of head_group whose K/V
        // fit in L2 together; inside a group causal blocks go heaviest first
        // across all its heads (src/fused/kernel.cpp:73,96), so the group's
        // K/V is read from HBM about once.
        const int mb = a.m_blocks;
        const int lin = blockIdx.x;
        const int g = lin / (a.head_group * mb);
        const int r = lin - g * a.head_group * mb;
        const int gs = min(a.head_group, a.num_hb - g * a.head_group);
        hb = g * a.head_group + r % gs;
        const int mrank = r / gs;
        mblk = kCausal ? mb - 1 - mrank : mrank;
    }
    // A list entry naming no (batch, head) of the problem, or a negative or
    // out-of-range query block, computes nothing and forms no address.
    if (hb < 0 || hb >= a.num_hb || mblk < 0 || mblk >= a.m_blocks) return false;
    w.h = hb % a.nhead_q;
    w.b = hb / a.nhead_q;
    w.kvh = w.h / (a.nhead_q / a.nhead_k);
    if constexpr (kVarlen) {
        // Full varlen launch: batch slots are walked longest sequence first.
        if (a.seq_order != nullptr && a.block_map == nullptr && a.tiles == nullptr &&
            a.items == nullptr)
            w.b = a.seq_order[w.b];
        w.off_q = a.seqstart_q[w.b];
        w.off_k = a.seqstart_k[w.b];
        w.seqlen_q = a.seqstart_q[w.b + 1] - w.off_q;
        w.seqlen_k = a.seqstart_k[w.b + 1] - w.off_k;
        if (w.off_q < 0 || w.off_k < 0 || w.seqlen_q < 0 || w.seqlen_k < 0 ||
            w.off_q + w.seqlen_q > a.total_q)
            return false;
    } else {
        w.off_q = 0;
        w.off_k = 0;
        w.seqlen_q = a.seqlen_q;
        w.seqlen_k = a.seqlen_k;
    }
    w.row0 = mblk * kRowsPerCta;
    if (w.row0 >= w.seqlen_q) return false;
    const int shift = w.seqlen_k - w.seqlen_q;  // bottom-right causal alignment
#pragma unroll
    for (int i = 0; i < kTilesPerCta; ++i) {
        const int r0 = w.row0 + i * kBlockM;
        if (r0 >= w.seqlen_q) {
            w.n_kv[i] = 0;
            continue;
        }
        int kv_end = w.seqlen_k;
        if (kCausal) {
            const int r_last = min(r0 + kBlockM - 1, w.seqlen_q - 1);
            kv_end = min(w.seqlen_k, r_last + shift + 1);
        }
        w.n_kv[i] = kv_end > 0 ? (kv_end + kBlockN - 1) / kBlockN : 0;
    }
    w.j0 = 0;
    w.partial = a.num_splits > 1 || (a.items != nullptr && kv_end >= 0);
    if (a.items != nullptr && kv_end >= 0) {
        const int jb = max(0, kv_begin);
#pragma unroll
        for (int i = 0; i < kTilesPerCta; ++i) w.n_kv[i] = max(0, min(w.n_kv[i], kv_end) - jb);
        w.j0 = jb;
    } else if (a.num_splits > 1) {
        // KV range of this split: an equal share of the longer tile's range.
        int n_all = 0;
#pragma unroll
        for (int i = 0; i < kTilesPerCta; ++i) n_all = max(n_all, w.n_kv[i]);
        const int chunk = (n_all + a.num_splits - 1) / a.num_splits;
        const int jb = split * chunk;
        const int je = min(n_all, jb + chunk);
        w.j0 = jb;
#pragma unroll
        for (int i = 0; i < kTilesPerCta; ++i) w.n_kv[i] = max(0, min(w.n_kv[i], je) - jb);
    }
    return true;
}

template <bool kVarlen>
__device__ __forceinline__ void tma_load_rows(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                              int row, int head, int batch, uint64_t policy) {
    if constexpr (kVarlen) {
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
            " [%0], [%1, {%2, %3, %4}], [%5], %6;"
            ::"r"(dst), "l"(tm), "r"(0), "r"(row), "r"(head), "r"(bar), "l"(policy)
            : "memory");
    } else {
        tma_load_4d(dst, tm, bar, 0, row, head, batch, policy);
    }
}

template <bool kCausal, bool kVarlen>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
fmha_fwd_d64_sm100_kernel(const __grid_constant__ KernelArgs a) {
    extern __shared__ uint8_t smem_raw[];
    SharedStorage& sm = *reinterpret_cast<SharedStorage*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    TileWork w;
    if (!decode_work<kCausal, kVarlen>(a, w)) return;  // CTA-uniform early out
    FMHA_TRACE_INIT;
    if (threadIdx.x == 0) FMHA_TRACE_CLOCK(7, 7);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    volatile int* abort_flag = &sm.abort_flag;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kTilesPerCta; ++i) {
            mbar_init(smem_u32(&sm.bar_q[i]), 1);
            mbar_init(smem_u32(&sm.bar_s[i]), 1);
            mbar_init(smem_u32(&sm.bar_sfree[i]), 32 * kWarpsPerTile);
            mbar_init(smem_u32(&sm.bar_p[i]), 32 * kWarpsPerTile);
            mbar_init(smem_u32(&sm.bar_pv[i]), 1);
            mbar_init(smem_u32(&sm.bar_o[i]), 1);
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&sm.bar_full[s]), 1);
            mbar_init(smem_u32(&sm.bar_empty[s]), 1);
        }
        mbar_init(smem_u32(&sm.bar_drain), 1);
        mbar_init(smem_u32(&sm.bar_dec), 32 * kSoftmaxWarps);
        sm.abort_flag = 0;
        sm.rerun = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(smem_u32(&sm.tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
        FMHA_TRACE_CLOCK(7, 0);
        FMHA_TRACE_AT(7, 1, smid());
    }
    const uint32_t tmem = sm.tmem_base;

    // Per-tile KV counts as scalars (a runtime-indexed array would live in
    // local memory).
    const int n_kv0 = w.n_kv[0];
    const int n_kv1 = kTilesPerCta > 1 ? w.n_kv[kTilesPerCta - 1] : 0;
    auto n_kv = [n_kv0, n_kv1](int i) { return i == 0 ? n_kv0 : n_kv1; };
    const int n_max = max(n_kv0, n_kv1);

    if (warp >= kSoftmaxWarps) {
    regs_dec<kRegsControl>();
    if (warp == kWarpLoad) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&a.tm_q);
            tma_prefetch_desc(&a.tm_k);
            tma_prefetch_desc(&a.tm_v);
            const uint64_t pol_q = l2_policy_evict_first();
            const uint64_t pol_kv = l2_policy_evict_last();
            const int qbatch = kVarlen ? 0 : w.b;
            for (int i = 0; i < kTilesPerCta; ++i) {
                if (n_kv(i) == 0) continue;
                const uint32_t bar = smem_u32(&sm.bar_q[i]);
                mbar_arrive_expect_tx(bar, kTileBytes);
                FMHA_TRACE_CLOCK(7, 5);
                tma_load_rows<kVarlen>(smem_u32(sm.q[i]), &a.tm_q, bar,
                                       w.off_q + w.row0 + i * kBlockM, w.h, qbatch, pol_q);
            }
            int issued = 0;  // loads issued into the ring
            bool ok = true;
            const int n_loads = 2 * n_max;
            // Pass 1 (the exact rerun, rare) streams the same K/V tiles again.
            for (int pass = 0; pass < 2 && ok && n_loads > 0; ++pass) {
            if (pass == 1) {
                if (!wait_phase(smem_u32(&sm.bar_dec), 0, abort_flag, a, kErrTimeoutLoad)) {
                    ok = false;
                    break;
                }
                if (!*reinterpret_cast<volatile int*>(&sm.rerun)) break;
            }
            for (int li = 0; li < n_loads; ++li) {
                const int idx = pass * n_loads + li;
                const int slot = idx % kStages;
                const uint32_t use = idx / kStages;
                if (!wait_phase(smem_u32(&sm.bar_empty[slot]), (use & 1) ^ 1, abort_flag, a,
                                kErrTimeoutLoad)) {
                    ok = false;
                    break;
                }
                if (a.stall_inject && idx == 1) {
                    // Test hook: never deliver V_0, so the MMA warp's wait runs
                    // out and the abort path is exercised without any fault.
                    continue;
                }
                const uint32_t bar = smem_u32(&sm.bar_full[slot]);
                mbar_arrive_expect_tx(bar, kTileBytes);
                const CUtensorMap* tm = (li & 1) ? &a.tm_v : &a.tm_k;
                tma_load_rows<kVarlen>(smem_u32(sm.kv[slot]), tm, bar,
                                       w.off_k + (w.j0 + (li >> 1)) * kBlockN, w.kvh,
                                       kVarlen ? 0 : w.b, pol_kv);
                issued = idx + 1;
                if (pass == 0) FMHA_TRACE_CLOCK(14 + (li & 1), li >> 1);
            }
            }
            if (!ok || *abort_flag) {
                // Let every copy this warp started land before the CTA exits.
                for (int i = 0; i < kTilesPerCta; ++i)
                    if (n_kv(i) > 0) drain_phase(smem_u32(&sm.bar_q[i]), 0, a);
                for (int idx = max(0, issued - kStages); idx < issued; ++idx) {
                    if (a.stall_inject && idx == 1) continue;
                    drain_phase(smem_u32(&sm.bar_full[idx % kStages]), (idx / kStages) & 1, a);
                }
            }
        }
        __syncwarp();
    } else if (warp == kWarpMma) {
        // ------------------------------------------------------ MMA issuer
        // The whole warp walks the schedule (waits included) so it stays
        // converged; one elected lane issues the tcgen05 instructions.  A
        // lone-lane issuer costs roughly 1.5-2x more cycles per MMA.
        const bool leader = elect_one();
        constexpr uint32_t idesc_qk = idesc_bf16_f32(kBlockM, kBlockN, 0, 0);
        constexpr uint32_t idesc_pv = idesc_bf16_f32(kBlockM, kHeadDim, 0, 1);
        const uint32_t kv_base = smem_u32(sm.kv[0]);
        // Descriptors are linear in the start address (bits 0-13 hold
        // address >> 4): each operand descriptor is a base descriptor plus a
        // byte offset >> 4.
        const uint64_t dq0 = smem_desc_sw128(smem_u32(sm.q[0]), 16, 1024);
        const uint64_t dk0 = smem_desc_sw128(kv_base, 16, 1024);
        const uint64_t dv0 = smem_desc_sw128(kv_base, 0, 1024);
        bool ok = true;

        auto slot_of = [](int idx) { return idx % kStages; };
        auto full_parity = [](int idx) { return (uint32_t)((idx / kStages) & 1); };
        auto wait_all = [&](uint64_t* bar, uint32_t parity) {
            const bool got = wait_phase(smem_u32(bar), parity, abort_flag, a, kErrTimeoutMma);
            return __all_sync(0xffffffffu, got);
        };
        auto commit = [&](uint64_t* bar) {
            if (leader) mma_commit(smem_u32(bar));
        };
        // S_i = Q_i K^T : M=128, N=128, K=64 as 4 x K16, 32 bytes (descriptor
        // +2) apart inside the 128-byte swizzled rows.
        auto issue_s = [&](int i, int slot) {
            const uint64_t da = dq0 + (uint64_t)(i * (kTileBytes >> 4));
            const uint64_t db = dk0 + (uint64_t)(slot * (kTileBytes >> 4));
            const uint32_t d = tmem + col_s(i);
            if (leader) {
                mma_ss(d, da, db, idesc_qk, 0u);
                mma_ss(d, da + 2, db + 2, idesc_qk, 1u);
                mma_ss(d, da + 4, db + 4, idesc_qk, 1u);
                mma_ss(d, da + 6, db + 6, idesc_qk, 1u);
            }
        };
        // O_i += P_i V : M=128, N=64, K=128 as 8 x K16.  P (bf16x2) is the
        // TMEM A operand; V is MN-major in shared memory, 16 keys = two 8-row
        // swizzle atoms = 2048 bytes (descriptor +128) per step.
        auto issue_pv = [&](int i, int slot, bool accumulate) {
            const uint64_t db = dv0 + (uint64_t)(slot * (kTileBytes >> 4));
            const uint32_t d = tmem + col_o(i);
            const uint32_t pa = tmem + col_p(i);
            if (leader) {
                mma_ts(d, pa, db, idesc_pv, accumulate ? 1u : 0u);
#pragma unroll
                for (int kk = 1; kk < kBlockN / 16; ++kk)
                    mma_ts(d, pa + kk * 8, db + (uint64_t)(kk * 128), idesc_pv, 1u);
            }
        };

        for (int i = 0; i < kTilesPerCta && ok; ++i)
            if (n_kv(i) > 0) ok = wait_all(&sm.bar_q[i], 0);
        if (leader) FMHA_TRACE_CLOCK(7, 6);
        // Pass 0 is the whole schedule; pass 1 (the exact rerun) repeats it
        // when the softmax asks for it, flat step index G + j.
        for (int pass = 0; pass < 2 && ok && n_max > 0; ++pass) {
        const int G = pass * n_max;
        if (pass == 1) {
            ok = wait_all(&sm.bar_dec, 0);
            if (!ok || !*reinterpret_cast<volatile int*>(&sm.rerun)) break;
            // S(G) overwrites S(G-1): the softmax has read it.
            ok = wait_all(&sm.bar_sfree[0], (G - 1) & 1);
            if (!ok) break;
        }
        ok = wait_all(&sm.bar_full[slot_of(2 * G)], full_parity(2 * G));
        if (ok) {
            tc_fence_after();
            for (int i = 0; i < kTilesPerCta; ++i) {
                if (n_kv(i) == 0) continue;
                issue_s(i, slot_of(2 * G));
                commit(&sm.bar_s[i]);
            }
            commit(&sm.bar_empty[slot_of(2 * G)]);
        }
        // Steady state, per KV tile j:
        //   S_i(j+1) as soon as softmax i has read S_i(j) (s_free) and K_{j+1}
        //   landed, then O_i += P_i(j) V_j once P_i(j) is written (p_full).
        for (int j = 0; j < n_max && ok; ++j) {
            const int g = G + j;
            const int v_idx = 2 * g + 1;
            const int k_idx = 2 * g + 2;
            bool k_used = false;
            for (int i = 0; i < kTilesPerCta; ++i) {
                if (j + 1 >= n_kv(i)) continue;
                if (!k_used) {
                    ok = wait_all(&sm.bar_full[slot_of(k_idx)], full_parity(k_idx));
                    if (leader && G == 0) FMHA_TRACE_CLOCK(8, j);
                    if (!ok) break;
                    k_used = true;
                }
                ok = wait_all(&sm.bar_sfree[i], g & 1);
                if (leader && G == 0) FMHA_TRACE_CLOCK(9, j);
                if (!ok) break;
                tc_fence_after();
                issue_s(i, slot_of(k_idx));
                if (leader && G == 0) FMHA_TRACE_CLOCK(5, j);
                commit(&sm.bar_s[i]);
            }
            if (!ok) break;
            if (k_used) commit(&sm.bar_empty[slot_of(k_idx)]);
            ok = wait_all(&sm.bar_full[slot_of(v_idx)], full_parity(v_idx));
            if (leader && G == 0) FMHA_TRACE_CLOCK(10, j);
            if (!ok) break;
            for (int i = 0; i < kTilesPerCta; ++i) {
                if (j >= n_kv(i)) continue;
                ok = wait_all(&sm.bar_p[i], g & 1);
                if (leader && G == 0) FMHA_TRACE_CLOCK(11, j);
                if (!ok) break;
                tc_fence_after();
                issue_pv(i, slot_of(v_idx), j > 0);
                if (leader && G == 0) FMHA_TRACE_CLOCK(6, j);
                commit(&sm.bar_pv[i]);
                if (j == n_kv(i) - 1) commit(&sm.bar_o[i]);
            }
            if (!ok) break;
            commit(&sm.bar_empty[slot_of(v_idx)]);
        }
        }
        // All MMAs this warp issued must finish before TMEM is freed.
        commit(&sm.bar_drain);
        drain_phase(smem_u32(&sm.bar_drain), 0, a);
        __syncwarp();
    }
#ifdef FMHA_TRACE
    else if (warp == kWarpMma + 1 && n_max > 0 && trace_row_ >= 0 &&
             trace_row_ < kTraceCtas) {
        // Trace builds only: an otherwise idle warp watches the MMA commits
        // of pass 0 and stamps when S(j) and PV(j) complete.
        // try_wait parks the warp until the phase completes (or its time
        // hint runs out), so the observer takes few issue slots.
        auto seen = [&](uint64_t* bar, uint32_t parity) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(smem_u32(bar), parity)) {
                if (*abort_flag || globaltimer_ns() - t0 > a.wait_limit_ns) return false;
            }
            return true;
        };
        if (seen(&sm.bar_s[0], 0) && lane == 0) FMHA_TRACE_CLOCK(12, 0);
        for (int j = 0; j < n_max; ++j) {
            if (j + 1 < n_max) {
                if (!seen(&sm.bar_s[0], (j + 1) & 1)) break;
                if (lane == 0) FMHA_TRACE_CLOCK(12, j + 1);
            }
            if (!seen(&sm.bar_pv[0], j & 1)) break;
            if (lane == 0) FMHA_TRACE_CLOCK(13, j);
        }
    }
#endif
    } else {
        regs_inc<kRegsSoftmax>();
        // ------------------------------------------------------ softmax groups
        const int i = warp >> 2;                    // query tile of this group
        const int t = threadIdx.x & (kBlockM - 1);  // row inside the tile == TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_base + col_s(i);
        const uint32_t tO = tmem + lane_base + col_o(i);
        const int n = n_kv(i);
        const int tile_row0 = w.row0 + i * kBlockM;
        const int row = tile_row0 + t;
        const int shift = w.seqlen_k - w.seqlen_q;
        const float scale = a.scale;
        // Keys visible to this row: [0, key_lim).
        const int key_lim = kCausal ? min(w.seqlen_k, row + shift + 1) : w.seqlen_k;

        float m_run = -INFINITY;  // un-scaled running max used as exp2 reference
        float l_run = 0.0f;       // running sum of un-normalised P
        bool ok = true;
        // Pass 0 ("fixed reference"): the exact row max of the first KV tile is
        // the exp2 reference for every later tile, so later tiles skip the row
        // max.  Any reference works as long as no P overflows: a later tile
        // whose row sum exceeds 2^40 (scores more than 40 log2 units above the
        // first tile's maximum) or a row with no visible key in the first tile
        // but some later flags the CTA, and pass 1 recomputes the query tile
        // with the exact running max (lazy rescale) -- rare, correct for any
        // input.
        int pass = 0;
        const int key_end0 = (w.j0 + 1) * kBlockN;  // keys of the first KV tile: [.., key_end0)

        const uint32_t tP = tmem + lane_base + col_p(i);
        // One pass over the KV tiles; fixed_tag selects the fixed-reference
        // variant at compile time, so each pass runs its own straight loop.
        // Returns whether a row outgrew the fixed reference.
        auto kv_pass = [&](auto fixed_tag) -> bool {
        constexpr bool fixed_ref = decltype(fixed_tag)::value;
        const int G = fixed_ref ? 0 : n;
        bool outgrown = false;
        m_run = -INFINITY;
        l_run = 0.0f;
        // One KV step; the first step of a pass is compiled separately
        // (first_tag), so the fixed-reference loop over the later steps carries
        // no row-max code at all.
        auto step = [&](int j, auto first_tag) -> bool {
            constexpr bool first = decltype(first_tag)::value;
            const int g = G + j;
            bool got = wait_phase(smem_u32(&sm.bar_s[i]), g & 1, abort_flag, a, kErrTimeoutSoftmax);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                return false;
            }
            tc_fence_after();
            if (fixed_ref && threadIdx.x == 0) FMHA_TRACE_CLOCK(0, j);
            uint32_t r[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, r[c]);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 4; ++c) reg_fence(r[c]);
            // S_i now lives in registers: the MMA warp may overwrite it with
            // S_i(j+1) while this group computes P_i(j).
            tc_fence_before();
            mbar_arrive(smem_u32(&sm.bar_sfree[i]));
            if (fixed_ref && threadIdx.x == 0) FMHA_TRACE_CLOCK(1, j);

            const int k0 = (w.j0 + j) * kBlockN;
            const bool need_mask = (k0 + kBlockN > w.seqlen_k) ||
                                   (kCausal && k0 + kBlockN - 1 > tile_row0 + shift);
            if (need_mask) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (k0 + c * 32 + e >= key_lim) r[c][e] = __float_as_uint(-INFINITY);
            }
            bool upd = false;
            float alpha = 1.0f;
            if (!fixed_ref || first) {
            // Row max: 8 independent 3-input-max chains.
            float mx[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) mx[q] = __uint_as_float(r[q >> 1][(q & 1) * 16]);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const uint32_t* rr = &r[q >> 1][(q & 1) * 16];
#pragma unroll
                for (int e = 1; e < 15; e += 2)
                    mx[q] = fmax3(mx[q], __uint_as_float(rr[e]), __uint_as_float(rr[e + 1]));
                mx[q] = fmaxf(mx[q], __uint_as_float(rr[15]));
            }
            const float row_max = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]),
                                        fmaxf(mx[6], mx[7]));
            const float m_new = fmaxf(m_run, row_max);
            upd = (m_new - m_run) * scale > kRescaleThreshold;
            if (upd) {
                alpha = ex2_approx((m_run - m_new) * scale);
                m_run = m_new;
            }
            if (fixed_ref && m_run == -INFINITY && key_lim > key_end0) outgrown = true;
            }
            const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
            const float neg_ms = kPLog2Bias - m_use * scale;
            const float2 scale2 = make_float2(scale, scale);
            const float2 neg2 = make_float2(neg_ms, neg_ms);
            float2 sum[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) sum[q] = make_float2(0.0f, 0.0f);
            uint32_t p[2][32];
            // P = exp2(S*scale - m*scale).  On tiles without masking a fixed
            // share of the pairs (kExpPolyPairs of every 16) runs the
            // polynomial exp2 on the FMA/ALU pipes, relieving MUFU; masked
            // tiles (which may hold -inf) use MUFU ex2 only.
            auto exp_tile = [&](auto poly_tag) {
                constexpr bool kPoly = decltype(poly_tag)::value;
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const int pr = e >> 1;  // pair index in the chunk
                        const float2 x = ffma2(make_float2(__uint_as_float(r[c][e]),
                                                           __uint_as_float(r[c][e + 1])),
                                               scale2, neg2);
                        float2 pp;
                        if (kPoly && ((pr + 1) * kExpPolyPairs / 16 > pr * kExpPolyPairs / 16))
                            pp = exp2_poly2(x);
                        else
                            pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                        sum[pr & 3] = fadd2(sum[pr & 3], pp);
                        p[c >> 1][(c & 1) * 16 + pr] = pack_bf16_trunc(pp.x, pp.y);
                    }
            };
            if (need_mask) exp_tile(std::false_type{});
            else exp_tile(std::true_type{});
            if (fixed_ref && threadIdx.x == 0) FMHA_TRACE_CLOCK(2, j);
            const float2 s01 = fadd2(fadd2(sum[0], sum[1]), fadd2(sum[2], sum[3]));
            const float tsum = s01.x + s01.y;
            l_run = fmaf(l_run, alpha, tsum);
            if (fixed_ref && !(tsum <= 0x1p40f)) outgrown = true;  // also catches inf / NaN

            if (g > 0) {
                // P_i(g-1) must be consumed (and O_i settled) before P_i(g) and the
                // O_i rescale are written.
                got = wait_phase(smem_u32(&sm.bar_pv[i]), (g - 1) & 1, abort_flag, a,
                                 kErrTimeoutSoftmax);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    return false;
                }
                tc_fence_after();
            }
            if (fixed_ref && threadIdx.x == 0) FMHA_TRACE_CLOCK(3, j);
            tmem_st32(tP, p[0]);
            tmem_st32(tP + 32, p[1]);
            if (j > 0 && __any_sync(0xffffffffu, upd)) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_wait_ld();
                    reg_fence(o);
                    const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float2 v2 = fmul2(make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), a2);
                        o[e] = __float_as_uint(v2.x);
                        o[e + 1] = __float_as_uint(v2.y);
                    }
                    tmem_st32(tO + c * 32, o);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(smem_u32(&sm.bar_p[i]));
            if (fixed_ref && threadIdx.x == 0) FMHA_TRACE_CLOCK(4, j);
                    return true;
        };
        if (n > 0 && step(0, std::true_type{})) {
            for (int j = 1; j < n; ++j)
                if (!step(j, std::false_type{})) break;
        }
        return outgrown;
        };
        const bool outgrown = kv_pass(std::true_type{});
        if (ok && n > 0) {
            // Verdict on pass 0, shared with the producer and MMA warps.
            if (__any_sync(0xffffffffu, outgrown) && lane == 0) atomicOr(&sm.rerun, 1);
            mbar_arrive(smem_u32(&sm.bar_dec));
            const bool got = wait_phase(smem_u32(&sm.bar_dec), 0, abort_flag, a, kErrTimeoutSoftmax);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
            } else if (*reinterpret_cast<volatile int*>(&sm.rerun)) {
                pass = 1;
                kv_pass(std::false_type{});
            }
        }

        // ---------------------------------------------------- epilogue
        // The merge launched after a split launch may be scheduled now: it
        // waits on the GPU for this grid to finish before reading anything.
        griddep_launch_dependents();
        if (ok && n > 0) {
            bool got = wait_phase(smem_u32(&sm.bar_o[i]), pass & 1, abort_flag, a,
                                  kErrTimeoutSoftmax);
            ok = __all_sync(0xffffffffu, got);
        }
        if (threadIdx.x == 0) FMHA_TRACE_CLOCK(7, 2);
        if (ok) {
            uint32_t o[2][32];
            if (n > 0) {
                tc_fence_after();
                tmem_ld32(tO, o[0]);
                tmem_ld32(tO + 32, o[1]);
                tmem_wait_ld();
                reg_fence(o[0]);
                reg_fence(o[1]);
            }
            if (w.partial) {
                // Split-KV: this item's normalised partial O (fp32) and LSE;
                // the combine kernel merges the splits of each query block.
                const float inv_l = (l_run > 0.0f) ? 1.0f / l_run : 0.0f;
                const size_t prow = (size_t)blockIdx.x * kRowsPerCta + (size_t)i * kBlockM + t;
                float4* dst = reinterpret_cast<float4*>(a.part_o + prow * kHeadDim);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    float v[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int col = c * 4 + e;
                        v[e] = n > 0 ? __uint_as_float(o[col >> 5][col & 31]) * inv_l : 0.0f;
                    }
                    dst[c] = make_float4(v[0], v[1], v[2], v[3]);
                }
                const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
                a.part_lse[prow] = (l_run > 0.0f)
                                       ? (__log2f(l_run) + m_use * scale - kPLog2Bias) *
                                             0.69314718055994531f
                                       : -INFINITY;
            } else if (row < w.seqlen_q) {
                const float inv_l = (l_run > 0.0f) ? 1.0f / l_run : 0.0f;
                uint16_t* orow;
                if constexpr (kVarlen) {
                    orow = a.o + (long long)w.h * a.nhead_stride_o +
                           (long long)(w.off_q + row) * a.stride_o;
                } else {
                    orow = a.o + (long long)w.b * a.batch_stride_o +
                           (long long)w.h * a.nhead_stride_o + (long long)row * a.stride_o;
                }
                uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int col = c * 8 + e * 2;
                        const float v0 = n > 0 ? __uint_as_float(o[col >> 5][col & 31]) * inv_l : 0.0f;
                        const float v1 = n > 0 ? __uint_as_float(o[(col + 1) >> 5][(col + 1) & 31]) * inv_l : 0.0f;
#ifdef FMHA_O_ROUND_TRUNC
                        pk[e] = pack_bf16_trunc(v0, v1);  // reference kernel's rounding
#else
                        pk[e] = pack_bf16_rne(v0, v1);
#endif
                    }
                    dst[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                if (a.lse != nullptr) {
                    const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
                    const float lse = (l_run > 0.0f)
                                          ? (__log2f(l_run) + m_use * scale - kPLog2Bias) *
                                                0.69314718055994531f
                                          : -INFINITY;
                    long long idx;
                    if constexpr (kVarlen) {
                        idx = (long long)w.h * a.total_q + w.off_q + row;
                    } else {
                        idx = ((long long)w.b * a.nhead_q + w.h) * a.seqlen_q + row;
                    }
                    a.lse[idx] = lse;
                }
            }
        }
        if (threadIdx.x == 0) FMHA_TRACE_CLOCK(7, 3);
}

    // ---------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) FMHA_TRACE_CLOCK(7, 4);
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}


// Varlen launch order: order[r] = the sequence of rank r when sequences are
// sorted by query length, longest first (ties by index), so the full-grid
// varlen launch deals the heaviest query blocks out first across
// sequences, not only inside one (src/fused/kernel.cpp:91-99 reverses the
// block index within a sequence).  One CTA; rank by counting.
__global__ void __launch_bounds__(1024)
fmha_fwd_d64_varlen_order(const int32_t* __restrict__ seqstart, int batch,
                          int32_t* __restrict__ order, int2* __restrict__ block_map,
                          int map_cap, int causal) {
    extern __shared__ int32_t lens[];
    __shared__ int warp_tot[32];
    for (int b = threadIdx.x; b < batch; b += blockDim.x) lens[b] = seqstart[b + 1] - seqstart[b];
    __syncthreads();
    for (int b = threadIdx.x; b < batch; b += blockDim.x) {
        const int lb = lens[b];
        int rank = 0;
        for (int c = 0; c < batch; ++c) {
            const int lc = lens[c];
            rank += (lc > lb) || (lc == lb && c < b);
        }
        order[rank] = b;
    }
    if (block_map == nullptr) return;
    __syncthreads();
    // Block map of the compact launch: position p of the rank-ordered list
    // of query blocks (longest sequence first; inside a sequence the
    // heaviest block first when causal) -> (sequence, query block).  Each
    // thread owns a contiguous run of ranks; an exclusive scan over the
    // threads' block counts gives where its run starts.
    const int seg = (batch + blockDim.x - 1) / blockDim.x;
    const int r0 = min(batch, (int)threadIdx.x * seg), r1 = min(batch, r0 + seg);
    auto nblk = [&](int r) { return (max(lens[order[r]], 0) + kBlockM - 1) / kBlockM; };
    int mine = 0;
    for (int r = r0; r < r1; ++r) mine += nblk(r);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int incl = mine;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        int t = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, t, d);
            if (lane >= d) t += v;
        }
        warp_tot[lane] = t;  // inclusive over warps
    }
    __syncthreads();
    int pos = incl - mine + (wid > 0 ? warp_tot[wid - 1] : 0);
    for (int r = r0; r < r1; ++r) {
        const int b = order[r];
        const int nb = nblk(r);
        for (int mi = 0; mi < nb && pos < map_cap; ++mi, ++pos)
            block_map[pos] = make_int2(b, causal ? nb - 1 - mi : mi);
    }
    // Positions past the last block (the grid is sized by an upper bound)
    // are marked empty.
    const int total = warp_tot[((blockDim.x + 31) >> 5) - 1];
    for (int q = total + (int)threadIdx.x; q < map_cap; q += blockDim.x)
        block_map[q] = make_int2(-1, -1);
}

// Split-KV merge: partial slots [slot0, slot0 + nparts) of query block mblk
// of (batch, head) hb -> O (bf16, rounded like the main epilogue) and LSE:
// LSE = log(sum_s exp(lse_s)), O = sum_s exp(lse_s - LSE) * O_s -- the LSE
// merge the reference's base-2 epilogue formula implies
// (src/fused/op_epilog.hpp:92-98).  A CTA of kCombineThreads merges
// kCombineRows rows of the block (quarter `part`): 16 threads per row, each
// owning 4 of the 64 columns, so a partial row is one coalesced 256-byte
// read and the splits' loads are independent.
constexpr int kCombineThreads = 512;
constexpr int kCombineRows = kCombineThreads / 16;          // 32 rows per CTA
constexpr int kCombineParts = kBlockM / kCombineRows;       // 4 CTAs per block

template <bool kVarlen>
__device__ __forceinline__ void merge_rows(const KernelArgs& a, int hb, int mblk, int slot0,
                                           int nparts, int part) {
    // Malformed list entries are skipped before any address is formed.
    if (hb < 0 || hb >= a.num_hb || mblk < 0 || mblk >= a.m_blocks) return;
    const int h = hb % a.nhead_q, b = hb / a.nhead_q;
    int seqlen_q = a.seqlen_q, off_q = 0;
    if constexpr (kVarlen) {
        off_q = a.seqstart_q[b];
        seqlen_q = a.seqstart_q[b + 1] - off_q;
        if (off_q < 0 || seqlen_q < 0 || off_q + seqlen_q > a.total_q) return;
    }
    const int r = part * kCombineRows + (int)(threadIdx.x >> 4);  // row inside the block
    const int c4 = threadIdx.x & 15;                              // float4 column group
    const int row = mblk * kBlockM + r;
    if (row >= seqlen_q) return;
    // Online merge in batches of kMergeBatch splits: the batch's LSEs and
    // partial rows are loaded together (independent loads in flight), then
    // folded into the running maximum / weight sum / accumulator.
    constexpr int kMergeBatch = 8;
    float mx = -INFINITY;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float wsum = 0.0f;
    for (int s0 = 0; s0 < nparts; s0 += kMergeBatch) {
        float l[kMergeBatch];
        float4 v[kMergeBatch];
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
            if (s0 + u < nparts) {
                const size_t prow = (size_t)(slot0 + s0 + u) * kBlockM + r;
                l[u] = a.part_lse[prow];
                v[u] = reinterpret_cast<const float4*>(a.part_o + prow * kHeadDim)[c4];
            } else {
                l[u] = -INFINITY;
                v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
        float mb = l[0];
#pragma unroll
        for (int u = 1; u < kMergeBatch; ++u) mb = fmaxf(mb, l[u]);
        const float mn = fmaxf(mx, mb);
        if (mn == -INFINITY) continue;  // no visible key in any split so far
        const float sc = __expf(mx - mn);  // 0 while mx is still -inf
        acc.x *= sc;
        acc.y *= sc;
        acc.z *= sc;
        acc.w *= sc;
        wsum *= sc;
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
            const float wgt = l[u] == -INFINITY ? 0.0f : __expf(l[u] - mn);
            wsum += wgt;
            acc.x += wgt * v[u].x;
            acc.y += wgt * v[u].y;
            acc.z += wgt * v[u].z;
            acc.w += wgt * v[u].w;
        }
        mx = mn;
    }
    const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
    uint16_t* orow;
    if constexpr (kVarlen) {
        orow = a.o + (long long)h * a.nhead_stride_o + (long long)(off_q + row) * a.stride_o;
    } else {
        orow = a.o + (long long)b * a.batch_stride_o + (long long)h * a.nhead_stride_o +
               (long long)row * a.stride_o;
    }
#ifdef FMHA_O_ROUND_TRUNC
    const uint2 pk = make_uint2(pack_bf16_trunc(acc.x * inv, acc.y * inv),
                                pack_bf16_trunc(acc.z * inv, acc.w * inv));
#else
    const uint2 pk = make_uint2(pack_bf16_rne(acc.x * inv, acc.y * inv),
                                pack_bf16_rne(acc.z * inv, acc.w * inv));
#endif
    reinterpret_cast<uint2*>(orow)[c4] = pk;
    if (a.lse != nullptr && c4 == 0) {
        const float lse = wsum > 0.0f ? mx + __logf(wsum) : -INFINITY;
        const long long idx = kVarlen ? (long long)h * a.total_q + off_q + row
                                      : ((long long)b * a.nhead_q + h) * a.seqlen_q + row;
        a.lse[idx] = lse;
    }
}

// Uniform split-KV combine: CTA (g, part) merges slots [g*S, g*S + S) of
// tiles[g], rows of quarter `part`.
template <bool kVarlen>
__global__ void __launch_bounds__(kCombineThreads)
fmha_fwd_d64_splitkv_combine(const __grid_constant__ KernelArgs a, int nblocks) {
    griddep_wait();  // the split launch has finished and its partials are visible
    const int item_block = blockIdx.x / kCombineParts;
    if (item_block >= nblocks) return;
    merge_rows<kVarlen>(a, a.tiles[2 * item_block], a.tiles[2 * item_block + 1],
                        item_block * a.num_splits, a.num_splits, blockIdx.x % kCombineParts);
}

// Work-item combine: CTA (x, part) merges the run of consecutive partial
// items of one query block that starts at item x (CTAs of other items return
// at once).  The run length is found with one parallel probe per thread
// (kCombineThreads items per pass), not a chain of dependent loads.
template <bool kVarlen>
__global__ void __launch_bounds__(kCombineThreads)
fmha_fwd_d64_items_combine(const __grid_constant__ KernelArgs a, int n_items) {
    __shared__ int run_end;
    griddep_wait();  // the split launch has finished and its partials are visible
    const int x = blockIdx.x / kCombineParts;
    const int4* items = reinterpret_cast<const int4*>(a.items);
    // A partial item has a well-formed KV range; malformed items were skipped
    // by the main kernel (no partial result) and take no part in any run.
    auto partial = [](const int4& e) { return e.w >= 0 && e.z >= 0 && e.z <= e.w; };
    const int4 it = items[x];
    if (!partial(it)) return;  // direct (O already written) or malformed item
    if (x > 0) {
        const int4 prev = items[x - 1];
        if (partial(prev) && prev.x == it.x && prev.y == it.y) return;  // not the run's head
    }
    int n = 0;
    for (int base = x + 1;; base += kCombineThreads) {
        if (threadIdx.x == 0) run_end = n_items;
        __syncthreads();
        const int y = base + (int)threadIdx.x;
        if (y < n_items) {
            const int4 nx = items[y];
            if (!partial(nx) || nx.x != it.x || nx.y != it.y) atomicMin(&run_end, y);
        }
        __syncthreads();
        const int e = run_end;
        __syncthreads();
        if (e < base + kCombineThreads || base + kCombineThreads >= n_items) {
            n = min(e, n_items) - x;
            break;
        }
    }
    merge_rows<kVarlen>(a, it.x, it.y, x, n, blockIdx.x % kCombineParts);
}

// ====================================================================== host

// Launch a merge kernel (KernelArgs, count) of kCombineThreads threads as a
// programmatic dependent of the previous launch on `stream`.
cudaError_t launch_dependent(void (*kern)(KernelArgs, int), dim3 grid, cudaStream_t stream,
                             const KernelArgs& a, int n) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kCombineThreads, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, n);
}

struct DeviceContext {
    bool ready = false;
    int* err_word = nullptr;
    // Varlen launch-order buffers, one per stream (launches on different
    // streams may overlap), grown on demand.
    std::vector<std::pair<cudaStream_t, std::pair<int32_t*, int>>> orders;
};

// Largest batch the varlen ordering handles (its one CTA ranks in shared
// memory); larger varlen launches keep the sequences' own order.
constexpr int kOrderMaxBatch = 8192;

std::mutex g_mutex;
std::vector<DeviceContext> g_devices;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
unsigned long long g_wait_limit_ns = 2000000000ull;
int g_stall_inject = 0;

constexpr size_t kSmemBytes = sizeof(SharedStorage) + 1024;

// Per-process, once: the driver's tensor-map encoder.  Caller holds g_mutex.
int ensure_encoder() {
    if (g_encode != nullptr) return FMHA_OK;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        fn == nullptr)
        return FMHA_ERR_DEVICE;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return FMHA_OK;
}

// Per device, once (device current): check it is an sm_100 part and set the
// kernels' shared-memory attributes.  Allocates nothing.
int prepare_device(int dev) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return FMHA_ERR_DEVICE;
    if (prop.major != 10 || prop.minor != 0) return FMHA_ERR_DEVICE;
    const int smem = (int)kSmemBytes;
    auto set = [smem](const void* fn) {
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    };
    set(reinterpret_cast<const void*>(fmha_fwd_d64_sm100_kernel<false, false>));
    set(reinterpret_cast<const void*>(fmha_fwd_d64_sm100_kernel<true, false>));
    set(reinterpret_cast<const void*>(fmha_fwd_d64_sm100_kernel<false, true>));
    set(reinterpret_cast<const void*>(fmha_fwd_d64_sm100_kernel<true, true>));
    return cudaGetLastError() == cudaSuccess ? FMHA_OK : FMHA_ERR_LAUNCH;
}

int ensure_context(int dev, DeviceContext** out) {
    std::lock_guard<std::mutex> lock(g_mutex);
    int st = ensure_encoder();
    if (st != FMHA_OK) return st;
    if ((int)g_devices.size() <= dev) g_devices.resize(dev + 1);
    DeviceContext& ctx = g_devices[dev];
    if (!ctx.ready) {
        if ((st = prepare_device(dev)) != FMHA_OK) return st;
        if (cudaMalloc(&ctx.err_word, sizeof(int)) != cudaSuccess) return FMHA_ERR_LAUNCH;
        if (cudaMemset(ctx.err_word, 0, sizeof(int)) != cudaSuccess) return FMHA_ERR_LAUNCH;
        ctx.ready = true;
    }
    *out = &ctx;
    return FMHA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Tensor map over a bf16 tensor seen as (d=64, rows, heads[, batch]), box of
// 64 x 128 rows, 128-byte swizzle (matches the UMMA SW128 canonical layout).
int make_map(CUtensorMap* tm, const uint16_t* base, int rank, int rows, int heads, int batch,
             long long row_stride, long long head_stride, long long batch_stride) {
    cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows, (cuuint64_t)heads,
                          (cuuint64_t)batch};
    // A stride of a size-1 dimension is never used; give it a legal value.
    if (heads == 1) head_stride = 8;
    if (batch == 1) batch_stride = 8;
    cuuint64_t strides[3] = {(cuuint64_t)row_stride * 2, (cuuint64_t)head_stride * 2,
                             (cuuint64_t)batch_stride * 2};
    cuuint32_t box[4] = {(cuuint32_t)kHeadDim, (cuuint32_t)kBlockM, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<uint16_t*>(base),
                          dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FMHA_OK : FMHA_ERR_ARG;
}

bool stride_ok(long long s, int extent) {
    if (extent <= 1) return true;
    return s > 0 && (s % 8) == 0 && s * 2 < (1ll << 40);
}

// Checks the problem description and fills everything of the kernel
// arguments except the work description, error word and launch options.
// Sets *empty when there is nothing to compute.
int prepare_args(const FmhaFwdParams* p, int batch, bool varlen, int total_q, int total_k,
                 KernelArgs& a, bool* empty) {
    *empty = false;
    if (p == nullptr || batch <= 0) return FMHA_ERR_ARG;
    if (!p->q || !p->k || !p->v || !p->o) return FMHA_ERR_ARG;
    if (p->nhead_q <= 0 || p->nhead_k <= 0 || p->nhead_q % p->nhead_k != 0) return FMHA_ERR_ARG;
    if (p->seqlen_q < 0 || p->seqlen_k < 0) return FMHA_ERR_ARG;
    if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->o))
        return FMHA_ERR_ARG;
    if (varlen) {
        if (!p->seqstart_q || !p->seqstart_k || total_q < 0 || total_k < 0) return FMHA_ERR_ARG;
    }
    const int rows_q = varlen ? total_q : p->seqlen_q;
    const int rows_k = varlen ? total_k : p->seqlen_k;
    if (!stride_ok(p->stride_q, rows_q) || !stride_ok(p->stride_k, rows_k) ||
        !stride_ok(p->stride_v, rows_k) || !stride_ok(p->nhead_stride_q, p->nhead_q) ||
        !stride_ok(p->nhead_stride_k, p->nhead_k) || !stride_ok(p->nhead_stride_v, p->nhead_k))
        return FMHA_ERR_ARG;
    if (!varlen && (!stride_ok(p->batch_stride_q, batch) || !stride_ok(p->batch_stride_k, batch) ||
                    !stride_ok(p->batch_stride_v, batch)))
        return FMHA_ERR_ARG;
    if ((p->stride_o % 8) != 0 || (p->nhead_stride_o % 8) != 0 ||
        (!varlen && (p->batch_stride_o % 8) != 0))
        return FMHA_ERR_ARG;
    if (p->seqlen_q == 0 || rows_q == 0) {
        *empty = true;
        return FMHA_OK;
    }
    const int m_blocks = (p->seqlen_q + kBlockM - 1) / kBlockM;
    if ((long long)m_blocks * p->nhead_q * batch > 0x7fffffffll) return FMHA_ERR_ARG;

    int st;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        if ((st = ensure_encoder()) != FMHA_OK) return st;
    }
    memset(&a, 0, sizeof(a));
    const int rank = varlen ? 3 : 4;
    const int mb = varlen ? 1 : batch;
    // K/V rows: a zero-length key sequence still needs a legal (1-row) map.
    const int rk = rows_k > 0 ? rows_k : 1;
    if ((st = make_map(&a.tm_q, p->q, rank, rows_q, p->nhead_q, mb, p->stride_q,
                       p->nhead_stride_q, p->batch_stride_q)) != FMHA_OK)
        return st;
    if ((st = make_map(&a.tm_k, p->k, rank, rk, p->nhead_k, mb, p->stride_k, p->nhead_stride_k,
                       p->batch_stride_k)) != FMHA_OK)
        return st;
    if ((st = make_map(&a.tm_v, p->v, rank, rk, p->nhead_k, mb, p->stride_v, p->nhead_stride_v,
                       p->batch_stride_v)) != FMHA_OK)
        return st;
    a.o = p->o;
    a.lse = p->lse;
    a.seqstart_q = varlen ? p->seqstart_q : nullptr;
    a.seqstart_k = varlen ? p->seqstart_k : nullptr;
    a.stride_o = p->stride_o;
    a.nhead_stride_o = p->nhead_stride_o;
    a.batch_stride_o = p->batch_stride_o;
    a.seqlen_q = p->seqlen_q;
    a.seqlen_k = p->seqlen_k;
    a.nhead_q = p->nhead_q;
    a.nhead_k = p->nhead_k;
    a.total_q = total_q;
    a.scale = p->scale;
    a.wait_limit_ns = g_wait_limit_ns;
    a.m_blocks = m_blocks;
    a.num_hb = p->nhead_q * batch;
    a.num_splits = 1;
    {
        // Group (batch, head) pairs so a group's K/V (read by all its blocks)
        // fits in ~48 MB of the 126 MB L2.
        const long long kv_bytes = (long long)p->seqlen_k * kHeadDim * 2 * 2;
        const long long g = kv_bytes > 0 ? (48ll << 20) / kv_bytes : a.num_hb;
        a.head_group = (int)std::max(1ll, std::min<long long>(g, a.num_hb));
    }
    return FMHA_OK;
}

// One CTA per work item (query tile, or split-KV item); CTAs start in work
// order, so the hardware hands the heaviest items out first.
int launch_main(const KernelArgs& a, bool causal, bool varlen, int n_work, cudaStream_t stream) {
    const unsigned grid = (unsigned)n_work;
    const dim3 block(kThreads);
    if (causal) {
        if (varlen) fmha_fwd_d64_sm100_kernel<true, true><<<grid, block, kSmemBytes, stream>>>(a);
        else fmha_fwd_d64_sm100_kernel<true, false><<<grid, block, kSmemBytes, stream>>>(a);
    } else {
        if (varlen) fmha_fwd_d64_sm100_kernel<false, true><<<grid, block, kSmemBytes, stream>>>(a);
        else fmha_fwd_d64_sm100_kernel<false, false><<<grid, block, kSmemBytes, stream>>>(a);
    }
    return cudaGetLastError() == cudaSuccess ? FMHA_OK : FMHA_ERR_LAUNCH;
}

int launch(const FmhaFwdParams* p, int batch, bool causal, bool varlen, int total_q, int total_k,
           cudaStream_t stream, const int32_t* tiles = nullptr, int ntiles = -1,
           int num_splits = 1, float* workspace = nullptr, const int32_t* items = nullptr,
           int n_items = 0) {
    KernelArgs a;
    bool empty = false;
    int st = prepare_args(p, batch, varlen, total_q, total_k, a, &empty);
    if (st != FMHA_OK || empty) return st;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_DEVICE;
    DeviceContext* ctx = nullptr;
    if ((st = ensure_context(dev, &ctx)) != FMHA_OK) return st;
    a.err_word = ctx->err_word;
    a.stall_inject = g_stall_inject;

    int n_work = a.m_blocks * a.num_hb;
    a.tiles = tiles;
    if (tiles != nullptr) {
        if (ntiles == 0) return FMHA_OK;
        n_work = ntiles;
        if (num_splits > 1) {
            a.num_splits = num_splits;
            a.part_o = workspace;
            a.part_lse = workspace + (size_t)ntiles * num_splits * kBlockM * kHeadDim;
            n_work = ntiles * num_splits;
        }
    }
    if (items != nullptr) {
        if (n_items == 0) return FMHA_OK;
        a.items = items;
        a.part_o = workspace;
        a.part_lse = workspace + (size_t)n_items * kBlockM * kHeadDim;
        n_work = n_items;
    }
    if (varlen && tiles == nullptr && items == nullptr && batch > 1 && batch <= kOrderMaxBatch) {
        // Compact launch: nhead_q CTAs per real query block (a sequence of
        // length L has ceil(L/128) blocks, at most total_q/128 + batch in
        // all), in the order of a block map built on the device, instead of
        // max-blocks x batch x heads CTAs of which the short sequences' tail
        // would exit at once.
        const long long cap_ll = std::min<long long>((long long)a.m_blocks * batch,
                                                     (long long)total_q / kBlockM + batch);
        const int cap = (int)cap_ll;
        const size_t order_ints = ((size_t)batch + 1) & ~(size_t)1;  // keeps the map 8-byte aligned
        const size_t need = order_ints + 2 * (size_t)cap;             // in int32 units
        int32_t* buf = nullptr;
        {
            std::lock_guard<std::mutex> lock(g_mutex);
            std::pair<int32_t*, int>* slot = nullptr;
            for (auto& e : ctx->orders)
                if (e.first == stream) slot = &e.second;
            if (slot == nullptr) {
                ctx->orders.push_back({stream, {nullptr, 0}});
                slot = &ctx->orders.back().second;
            }
            if ((size_t)slot->second < need) {
                if (slot->first) cudaFree(slot->first);
                slot->first = nullptr;
                slot->second = 0;
                if (cudaMalloc(&slot->first, sizeof(int32_t) * need) != cudaSuccess)
                    return FMHA_ERR_LAUNCH;
                slot->second = (int)need;
            }
            buf = slot->first;
        }
        int2* map = reinterpret_cast<int2*>(buf + order_ints);
        fmha_fwd_d64_varlen_order<<<1, 1024, sizeof(int32_t) * (size_t)batch, stream>>>(
            p->seqstart_q, batch, buf, map, cap, causal ? 1 : 0);
        a.seq_order = buf;
        a.block_map = map;
        n_work = cap * p->nhead_q;
    }
    if ((st = launch_main(a, causal, varlen, n_work, stream)) != FMHA_OK)
        return st;
    // The merge goes out with programmatic stream serialization, so its
    // launch overlaps the split launch's tail (see griddep_wait).
    if (items != nullptr) {
        const dim3 cgrid((unsigned)(n_items * kCombineParts), 1, 1);
        if (launch_dependent(varlen ? fmha_fwd_d64_items_combine<true>
                                    : fmha_fwd_d64_items_combine<false>,
                             cgrid, stream, a, n_items) != cudaSuccess)
            return FMHA_ERR_LAUNCH;
    } else if (a.num_splits > 1) {
        const dim3 cgrid((unsigned)(ntiles * kCombineParts), 1, 1);
        if (launch_dependent(varlen ? fmha_fwd_d64_splitkv_combine<true>
                                    : fmha_fwd_d64_splitkv_combine<false>,
                             cgrid, stream, a, ntiles) != cudaSuccess)
            return FMHA_ERR_LAUNCH;
    }
    return cudaGetLastError() == cudaSuccess ? FMHA_OK : FMHA_ERR_LAUNCH;
}

}  // namespace

// ============================================ allocation-free variant (host)
//
// For callers that may not allocate device memory themselves -- for example
// code that runs where a cudaMalloc would be refused or would stall the whole
// device (inside a stream capture, or a serving loop that must never
// synchronise), or a plug-in whose host framework owns every allocation.  The
// regular entries allocate a small per-device error word on their first call;
// this variant instead keeps its scratch (the error word and a staged copy of
// the caller's work list) in the file-scope array below, which every GPU that
// loads the library holds until the process exits.
namespace {

constexpr int kNoAllocMaxTiles = 16384;     // work-list capacity (query blocks)
constexpr int kNoAllocHeaderInts = 64;      // [0] = device error word
static __device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocHeaderInts + 2 * kNoAllocMaxTiles];

struct NoAllocDevice {
    bool ready = false;
    int32_t* scratch = nullptr;  // device address of g_noalloc_scratch on that device
};
std::vector<NoAllocDevice> g_noalloc;

// Once per device, with that device current: resolve the device address of
// the scratch array (the host-side name is only a stand-in) and set the
// kernels' shared-memory attribute.  Allocates nothing.
int noalloc_setup(int dev, NoAllocDevice** out) {
    std::lock_guard<std::mutex> lock(g_mutex);
    int st = ensure_encoder();
    if (st != FMHA_OK) return st;
    if ((int)g_noalloc.size() <= dev) g_noalloc.resize(dev + 1);
    NoAllocDevice& d = g_noalloc[dev];
    if (!d.ready) {
        if ((st = prepare_device(dev)) != FMHA_OK) return st;
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
            return FMHA_ERR_LAUNCH;
        d.scratch = static_cast<int32_t*>(ptr);
        d.ready = true;
    }
    *out = &d;
    return FMHA_OK;
}

int launch_noalloc(const FmhaFwdParams* p, int batch, bool causal, int total_q, int total_k,
                   const int32_t* host_tiles, int ntiles, cudaStream_t stream) {
    if (p == nullptr || batch <= 0 || ntiles < 0) return FMHA_ERR_ARG;
    if (ntiles > kNoAllocMaxTiles) return FMHA_ERR_SCRATCH;
    if (ntiles > 0 && host_tiles == nullptr) return FMHA_ERR_ARG;
    const bool varlen = p->seqstart_q != nullptr;
    // The list is on the host, so every entry is checked before anything is
    // queued: a (batch, head) index or query block outside the problem is an
    // argument error, not a silent skip.
    if (p->nhead_q <= 0 || p->seqlen_q < 0) return FMHA_ERR_ARG;
    const long long num_hb = (long long)p->nhead_q * batch;
    const int m_blocks = (p->seqlen_q + kBlockM - 1) / kBlockM;
    for (int i = 0; i < ntiles; ++i) {
        const int32_t hb = host_tiles[2 * i], m = host_tiles[2 * i + 1];
        if (hb < 0 || hb >= num_hb || m < 0 || m >= m_blocks) return FMHA_ERR_ARG;
    }
    KernelArgs a;
    bool empty = false;
    int st = prepare_args(p, batch, varlen, total_q, total_k, a, &empty);
    if (st != FMHA_OK) return st;
    if (ntiles == 0 || empty) return FMHA_OK;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_DEVICE;
    NoAllocDevice* d = nullptr;
    if ((st = noalloc_setup(dev, &d)) != FMHA_OK) return st;
    int32_t* scratch = d->scratch;
    a.err_word = scratch;  // header word 0
    a.stall_inject = 0;
    a.tiles = scratch + kNoAllocHeaderInts;

    // The array keeps the previous call's contents: clear the error word and
    // stage this call's work list, in stream order before the kernel.
    if (cudaMemsetAsync(scratch, 0, sizeof(int32_t), stream) != cudaSuccess) return FMHA_ERR_LAUNCH;
    if (cudaMemcpyAsync(scratch + kNoAllocHeaderInts, host_tiles,
                        sizeof(int32_t) * 2 * (size_t)ntiles, cudaMemcpyHostToDevice,
                        stream) != cudaSuccess)
        return FMHA_ERR_LAUNCH;
    return launch_main(a, causal, varlen, ntiles, stream);
}

// Reads the error word of the allocation-free scratch and clears it, so a
// second status call (or one after a later failed launch) does not report a
// stale timeout.
int noalloc_status(cudaStream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_DEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return FMHA_ERR_LAUNCH;
    int32_t* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        if (dev < (int)g_noalloc.size() && g_noalloc[dev].ready) scratch = g_noalloc[dev].scratch;
    }
    if (scratch == nullptr) return FMHA_OK;
    int h = 0;
    if (cudaMemcpy(&h, scratch, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return FMHA_ERR_LAUNCH;
    if (h != 0) {
        if (cudaMemsetAsync(scratch, 0, sizeof(int32_t), stream) != cudaSuccess ||
            cudaStreamSynchronize(stream) != cudaSuccess)
            return FMHA_ERR_LAUNCH;
        return FMHA_ERR_TIMEOUT;
    }
    return FMHA_OK;
}

}  // namespace

#ifdef FMHA_TRACE
// Trace-build entry points (include/fmha_fwd_trace.h).
extern "C" {
int fmha_fwd_d64_trace_shape(int* ctas, int* steps, int* slots) {
    if (!ctas || !steps || !slots) return FMHA_ERR_ARG;
    *ctas = kTraceCtas;
    *steps = kTraceSteps;
    *slots = kTraceSlots;
    return FMHA_OK;
}
int fmha_fwd_d64_trace_configure(int first_cta) {
    if (first_cta < 0) return FMHA_ERR_ARG;
    void* buf = nullptr;
    if (cudaMemcpyToSymbol(g_trace_cta0, &first_cta, sizeof(int)) != cudaSuccess ||
        cudaGetSymbolAddress(&buf, g_trace) != cudaSuccess ||
        cudaMemset(buf, 0, sizeof(unsigned long long) * kTraceCtas * kTraceSteps * kTraceSlots) !=
            cudaSuccess)
        return FMHA_ERR_DEVICE;
    return FMHA_OK;
}
int fmha_fwd_d64_trace_read(unsigned long long* dst, size_t count) {
    if (!dst || count > (size_t)kTraceCtas * kTraceSteps * kTraceSlots) return FMHA_ERR_ARG;
    return cudaMemcpyFromSymbol(dst, g_trace, count * sizeof(unsigned long long)) == cudaSuccess
               ? FMHA_OK
               : FMHA_ERR_DEVICE;
}
}  // extern "C"
#endif

extern "C" {

int fmha_fwd_d64_bf16_msk0(const FmhaFwdParams* params, int batch, CUstream_st* stream) {
    if (params && (params->seqstart_q || params->seqstart_k)) return FMHA_ERR_ARG;
    return launch(params, batch, false, false, 0, 0, stream);
}
int fmha_fwd_d64_bf16_msk1(const FmhaFwdParams* params, int batch, CUstream_st* stream) {
    if (params && (params->seqstart_q || params->seqstart_k)) return FMHA_ERR_ARG;
    return launch(params, batch, true, false, 0, 0, stream);
}
int fmha_fwd_d64_bf16_msk0_varlen(const FmhaFwdParams* params, int batch, int total_q,
                                  int total_k, CUstream_st* stream) {
    return launch(params, batch, false, true, total_q, total_k, stream);
}
int fmha_fwd_d64_bf16_msk1_varlen(const FmhaFwdParams* params, int batch, int total_q,
                                  int total_k, CUstream_st* stream) {
    return launch(params, batch, true, true, total_q, total_k, stream);
}
int fmha_fwd_d64_bf16(const FmhaFwdParams* params, int batch, int causal, int total_q,
                      int total_k, CUstream_st* stream) {
    if (params == nullptr) return FMHA_ERR_ARG;
    const bool varlen = params->seqstart_q != nullptr;
    return launch(params, batch, causal != 0, varlen, total_q, total_k, stream);
}

int fmha_fwd_d64_bf16_tiles(const FmhaFwdParams* params, int batch, int causal, int total_q,
                            int total_k, const int32_t* tiles, int ntiles, CUstream_st* stream) {
    if (params == nullptr || ntiles < 0) return FMHA_ERR_ARG;
    if (ntiles == 0) return FMHA_OK;  // nothing to compute (tiles may be NULL)
    if (tiles == nullptr) return FMHA_ERR_ARG;
    if (((uintptr_t)tiles & 7u) != 0) return FMHA_ERR_ARG;
    const bool varlen = params->seqstart_q != nullptr;
    return launch(params, batch, causal != 0, varlen, total_q, total_k, stream, tiles, ntiles);
}

int fmha_fwd_d64_rows_per_block(void) { return kBlockM; }

size_t fmha_fwd_d64_splitkv_workspace_bytes(int ntiles, int num_splits) {
    if (ntiles <= 0 || num_splits <= 0) return 0;
    return (size_t)ntiles * num_splits * kBlockM * (kHeadDim + 1) * sizeof(float);
}

int fmha_fwd_d64_bf16_tiles_splitkv(const FmhaFwdParams* params, int batch, int causal,
                                    int total_q, int total_k, const int32_t* tiles, int ntiles,
                                    int num_splits, void* workspace, size_t workspace_bytes,
                                    CUstream_st* stream) {
    if (params == nullptr || ntiles < 0 || num_splits < 1 || num_splits > 64) return FMHA_ERR_ARG;
    if (ntiles == 0) return FMHA_OK;
    if (tiles == nullptr || ((uintptr_t)tiles & 7u) != 0) return FMHA_ERR_ARG;
    if (num_splits == 1)
        return launch(params, batch, causal != 0, params->seqstart_q != nullptr, total_q, total_k,
                      stream, tiles, ntiles);
    if (workspace == nullptr || ((uintptr_t)workspace & 15u) != 0 ||
        workspace_bytes < fmha_fwd_d64_splitkv_workspace_bytes(ntiles, num_splits))
        return FMHA_ERR_ARG;
    if ((long long)ntiles * num_splits > 0x7fffffffll) return FMHA_ERR_ARG;
    return launch(params, batch, causal != 0, params->seqstart_q != nullptr, total_q, total_k,
                  stream, tiles, ntiles, num_splits, static_cast<float*>(workspace));
}

size_t fmha_fwd_d64_items_workspace_bytes(int n_items) {
    if (n_items <= 0) return 0;
    return (size_t)n_items * kBlockM * (kHeadDim + 1) * sizeof(float);
}

int fmha_fwd_d64_bf16_items(const FmhaFwdParams* params, int batch, int causal, int total_q,
                            int total_k, const int32_t* items, int n_items, void* workspace,
                            size_t workspace_bytes, CUstream_st* stream) {
    if (params == nullptr || n_items < 0) return FMHA_ERR_ARG;
    if (n_items == 0) return FMHA_OK;
    if (items == nullptr || ((uintptr_t)items & 15u) != 0) return FMHA_ERR_ARG;
    if (workspace == nullptr || ((uintptr_t)workspace & 15u) != 0 ||
        workspace_bytes < fmha_fwd_d64_items_workspace_bytes(n_items))
        return FMHA_ERR_ARG;
    return launch(params, batch, causal != 0, params->seqstart_q != nullptr, total_q, total_k,
                  stream, nullptr, -1, 1, static_cast<float*>(workspace), items, n_items);
}

int fmha_fwd_d64_status(CUstream_st* stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_DEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return FMHA_ERR_LAUNCH;
    int* word = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        if (dev < (int)g_devices.size() && g_devices[dev].ready) word = g_devices[dev].err_word;
    }
    if (word == nullptr) return FMHA_OK;
    int h = 0;
    if (cudaMemcpy(&h, word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return FMHA_ERR_LAUNCH;
    if (h != 0) {
        cudaMemset(word, 0, sizeof(int));
        return FMHA_ERR_TIMEOUT;
    }
    return FMHA_OK;
}

void fmha_fwd_d64_set_wait_limit_ns(unsigned long long limit_ns) {
    std::lock_guard<std::mutex> lock(g_mutex);
    g_wait_limit_ns = limit_ns ? limit_ns : 2000000000ull;
}

// Test hook (not in the public header's main API): makes the producer warp
// withhold the first V tile so the bounded waits expire.  Used only by the
// timeout test, which also shortens the wait limit.
void fmha_fwd_d64_debug_set_stall(int enable) {
    std::lock_guard<std::mutex> lock(g_mutex);
    g_stall_inject = enable;
}

void fmha_fwd_d64_release(void) {
    std::lock_guard<std::mutex> lock(g_mutex);
    int cur = 0;
    cudaGetDevice(&cur);
    for (size_t d = 0; d < g_devices.size(); ++d) {
        if (g_devices[d].ready) {
            cudaSetDevice((int)d);
            cudaFree(g_devices[d].err_word);
            for (auto& e : g_devices[d].orders) cudaFree(e.second.first);
            g_devices[d] = DeviceContext();
        }
    }
    cudaSetDevice(cur);
}

int fmha_fwd_d64_bf16_tiles_noalloc(const FmhaFwdParams* params, int batch, int causal,
                                    int total_q, int total_k, const int32_t* host_tiles,
                                    int ntiles, CUstream_st* stream) {
    return launch_noalloc(params, batch, causal != 0, total_q, total_k, host_tiles, ntiles,
                          stream);
}

int fmha_fwd_d64_noalloc_status(CUstream_st* stream) { return noalloc_status(stream); }

const char* fmha_fwd_d64_error_string(int status) {
    switch (status) {
        case FMHA_OK: return "ok";
        case FMHA_ERR_ARG: return "invalid argument";
        case FMHA_ERR_LAUNCH: return "CUDA launch or runtime error";
        case FMHA_ERR_TIMEOUT: return "device pipeline wait exceeded its time limit";
        case FMHA_ERR_DEVICE: return "no supported sm_100 device";
        case FMHA_ERR_SCRATCH:
            return "work list longer than the allocation-free entry's scratch (16384 blocks)";
        default: return "unknown status";
    }
}

}  // extern "C"
