// fmha_fwd_kernel.cu -- B200 (sm_100a) head-dim-64 BF16 fused attention
// forward, and the C-ABI launchers declared in include/fmha_fwd.h.
//
// A persistent CTA loops over 128-row query tiles of (batch, head) pairs
// (work items dealt out in rounds, alternating direction) and walks each
// tile's key/value sequence in 128-key tiles; two CTAs share each SM, each
// with its own pipeline.  The CTA is warp specialised:
//
//   warps 0-3  softmax + epilogue : one query row per thread (TMEM lane = row)
//   warp  4    TMA producer       : Q of the current and next tile (double
//                                   buffer), K_j / V_j into a 4-slot ring
//   warp  5    MMA issuer         : one elected lane issues every tcgen05.mma;
//                                   the warp also owns the TMEM allocation
//   warps 6-7  idle               : complete the control warpgroup for setmaxnreg
//
// Tensor memory (256 columns x 128 lanes per CTA; two CTAs fill the SM):
//   [  0,128) S = Q K^T (fp32)
//   [128,192) O accumulator (fp32)
//   [192,256) P (bf16x2)
//
// The pipeline is one flat stream of KV steps g across the CTA's tiles:
//   MMA : S(g) = Q K^T -> commit(s_full)
//   SM  : S -> registers -> arrive(s_free) -> mask, row max, (lazy) rescale
//         of O -> P = exp2(S*scale - m*scale) -> wait(pv_done(g-1)) ->
//         bf16 P into TMEM -> arrive(p_full)
//   MMA : S(g+1) as soon as s_free arrives (also when g+1 starts the next
//         tile), then O += P(g) V(g) -> commit(pv_done)
//   SM  : after a tile's last step: wait(pv_done), O -> registers ->
//         arrive(o_free) -> O/l and LSE to global memory; the MMA warp starts
//         the next tile's first P V only after o_free.
// tcgen05 MMAs issued by one thread execute in order, so pv_done(g-1) also
// proves every earlier MMA finished, which is what makes the softmax-side O
// rescale race free.
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
constexpr int kCtasPerSm = 2;           // two independent persistent CTAs per SM
constexpr int kStages = 4;              // K/V ring slots (K_j, V_j alternate)
constexpr int kTileBytes = kBlockM * kHeadDim * 2;  // 16 KB (Q, K or V tile)
constexpr int kSoftmaxWarps = 4;        // one thread per query row
constexpr int kThreads = 32 * kSoftmaxWarps + 128;  // softmax group + control group
// Register split (setmaxnreg): the CTA launches with kThreads x kLaunchRegs
// registers; the softmax group takes kRegsSoftmax, the producer/MMA group
// kRegsControl: 128 * (192 + 64) <= 256 * 128.
constexpr int kRegsSoftmax = 192;
constexpr int kRegsControl = 64;
constexpr int kLaunchRegs = 128;
static_assert(128 * kRegsSoftmax + 128 * kRegsControl <= kThreads * kLaunchRegs,
              "setmaxnreg split exceeds the launch register pool");
constexpr int kWarpLoad = kSoftmaxWarps;
constexpr int kWarpMma = kSoftmaxWarps + 1;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0;    // S = Q K^T (fp32), 128 columns
constexpr uint32_t kColO = 128;  // O accumulator (fp32), 64 columns
constexpr uint32_t kColP = 192;  // P (bf16x2), 64 columns
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

struct KernelArgs {
    CUtensorMap tm_q;
    CUtensorMap tm_k;
    CUtensorMap tm_v;
    uint16_t* o;
    float* lse;
    const int32_t* seqstart_q;
    const int32_t* seqstart_k;
    long long stride_o, nhead_stride_o, batch_stride_o;
    int seqlen_q, seqlen_k;
    int nhead_q, nhead_k;
    int total_q;               // varlen: LSE head stride
    float scale;
    int* err_word;
    unsigned long long wait_limit_ns;
    int stall_inject;          // test hook: producer withholds the first V tile
    int n_work;                // work items of the launch (CTAs loop over them)
    const int32_t* tiles;      // optional work list of (b*nhead_q+h, query block)
    int m_blocks;              // query blocks per (batch, head) in a full launch
    int head_group;            // (batch, head) pairs per L2 group of the launch order
    int num_hb;                // batch * nhead_q
    int num_splits;            // split-KV: work item x = (tiles[x / num_splits], KV range x % num_splits)
    const int32_t* items;      // optional work items (b*nhead_q+h, query block, kv_begin, kv_end)
    float* part_o;             // split-KV partial O (fp32, normalised) [item][128][64]
    float* part_lse;           // split-KV partial LSE (natural log) [item][128]
};

struct TileWork {
    int n;                      // KV tiles the query tile walks (from j0)
    int j0;                     // first KV tile (split-KV ranges start past 0)
    int row0;                   // first query row of the tile (sequence-local)
    int seqlen_q, seqlen_k;
    int off_q, off_k;           // varlen packed-row offsets
    int b, h, kvh;
    int x;                      // work-item index (split-KV workspace slot)
    bool partial;               // split-KV item: partial O/LSE into the workspace
};

struct alignas(1024) SharedStorage {
    uint8_t q[2][kTileBytes];      // Q of the current and the next query tile
    uint8_t kv[kStages][kTileBytes];
    uint64_t bar_qfull[2];
    uint64_t bar_qempty[2];        // Q buffer's last S issued and done (MMA commit)
    uint64_t bar_full[kStages];
    uint64_t bar_empty[kStages];
    uint64_t bar_s;                // S written (MMA commit)
    uint64_t bar_sfree;            // S read into registers (128 arrivals)
    uint64_t bar_p;                // P written, O rescaled (128 arrivals)
    uint64_t bar_pv;               // O += P V done (MMA commit)
    uint64_t bar_ofree;            // final O of a tile read out (128 arrivals)
    uint64_t bar_drain;
    TileWork work[kSoftmaxWarps];  // softmax warps' current tile (see the softmax loop)
    uint32_t tmem_base;
    int abort_flag;
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


// Work item x of the launch -> query tile and KV range.  Returns false for an
// item that computes nothing (a query block past the end of its sequence,
// or a malformed work-list entry, which is skipped without any access).
template <bool kCausal, bool kVarlen>
__device__ __forceinline__ bool decode_work(const KernelArgs& a, int x, TileWork& w) {
    int hb, mblk;
    int split = 0;
    int kv_begin = 0, kv_end = -1;  // work items: explicit KV-tile range (end < 0: all)
    if (a.items != nullptr) {
        const int4 it = reinterpret_cast<const int4*>(a.items)[x];
        hb = it.x;
        mblk = it.y;
        kv_begin = it.z;
        kv_end = it.w;
        if (kv_end >= 0 && (kv_begin < 0 || kv_begin > kv_end)) return false;
    } else if (a.tiles != nullptr) {
        // Caller-supplied work list: (batch*nhead_q + head, query block); in
        // split-KV mode every entry expands into num_splits KV ranges.
        const int e = a.num_splits > 1 ? x / a.num_splits : x;
        if (a.num_splits > 1) split = x - e * a.num_splits;
        hb = a.tiles[2 * e];
        mblk = a.tiles[2 * e + 1];
    } else {
        // Launch order: (batch, head) pairs in groups of head_group whose K/V
        // fit in L2 together; inside a group causal blocks go heaviest first
        // across all its heads (src/fused/kernel.cpp:73,96), so the group's
        // K/V is read from HBM about once.
        const int mb = a.m_blocks;
        const int g = x / (a.head_group * mb);
        const int r = x - g * a.head_group * mb;
        const int gs = min(a.head_group, a.num_hb - g * a.head_group);
        hb = g * a.head_group + r % gs;
        const int mrank = r / gs;
        mblk = kCausal ? mb - 1 - mrank : mrank;
    }
    // A list entry naming no (batch, head) of the problem, or a negative or
    // out-of-range query block, is skipped before any address is formed.
    if (hb < 0 || hb >= a.num_hb || mblk < 0 || mblk >= a.m_blocks) return false;
    w.x = x;
    w.h = hb % a.nhead_q;
    w.b = hb / a.nhead_q;
    w.kvh = w.h / (a.nhead_q / a.nhead_k);
    if constexpr (kVarlen) {
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
    w.row0 = mblk * kBlockM;
    if (w.row0 >= w.seqlen_q) return false;
    const int shift = w.seqlen_k - w.seqlen_q;  // bottom-right causal alignment
    int kend = w.seqlen_k;
    if (kCausal) {
        const int r_last = min(w.row0 + kBlockM - 1, w.seqlen_q - 1);
        kend = min(w.seqlen_k, r_last + shift + 1);
    }
    w.n = kend > 0 ? (kend + kBlockN - 1) / kBlockN : 0;
    w.j0 = 0;
    w.partial = a.num_splits > 1 || (a.items != nullptr && kv_end >= 0);
    if (a.items != nullptr && kv_end >= 0) {
        w.n = max(0, min(w.n, kv_end) - kv_begin);
        w.j0 = kv_begin;
    } else if (a.num_splits > 1) {
        // KV range of this split: an equal share of the tile's range.
        const int chunk = (w.n + a.num_splits - 1) / a.num_splits;
        const int jb = split * chunk;
        const int je = min(w.n, jb + chunk);
        w.j0 = jb;
        w.n = max(0, je - jb);
    }
    return true;
}

// k-th work item of this CTA: items are dealt out in rounds of gridDim.x,
// alternately in CTA order and in reverse ("snake"), so a list sorted
// heaviest first spreads its heavy and light items evenly over the CTAs.
// Returns -1 past the end of the list, -2 for a hole in the last round.
__device__ __forceinline__ int work_index(const KernelArgs& a, int k) {
    const int g = (int)gridDim.x;
    const long long base = (long long)k * g;
    if (base >= a.n_work) return -1;
    const int c = (int)blockIdx.x;
    const long long x = base + ((k & 1) ? (g - 1 - c) : c);
    return x < a.n_work ? (int)x : -2;
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

// Output of one query row: O * (1/l) rounded to bf16 and the LSE (dense or
// varlen layouts), or for a split-KV item the normalised fp32 partial O and
// its LSE in the workspace.  `o` holds the row's 64 fp32 accumulator columns
// (zeros when the tile visited no key: the row is O = 0, LSE = -inf,
// src/fused/pipeline.hpp:207-222).
template <bool kVarlen>
__device__ __forceinline__ void store_row(const KernelArgs& a, const TileWork& w, int t,
                                          const uint32_t (&o)[2][32], bool any_key, float m_run,
                                          float l_run) {
    const int row = w.row0 + t;
    const float inv_l = (any_key && l_run > 0.0f) ? 1.0f / l_run : 0.0f;
    const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
    const float lse = (any_key && l_run > 0.0f)
                          ? (__log2f(l_run) + m_use * a.scale - kPLog2Bias) * 0.69314718055994531f
                          : -INFINITY;
    if (w.partial) {
        const size_t prow = (size_t)w.x * kBlockM + t;
        float4* dst = reinterpret_cast<float4*>(a.part_o + prow * kHeadDim);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = c * 4 + e;
                v[e] = __uint_as_float(o[col >> 5][col & 31]) * inv_l;
            }
            dst[c] = make_float4(v[0], v[1], v[2], v[3]);
        }
        a.part_lse[prow] = lse;
        return;
    }
    if (row >= w.seqlen_q) return;
    uint16_t* orow;
    if constexpr (kVarlen) {
        orow = a.o + (long long)w.h * a.nhead_stride_o + (long long)(w.off_q + row) * a.stride_o;
    } else {
        orow = a.o + (long long)w.b * a.batch_stride_o + (long long)w.h * a.nhead_stride_o +
               (long long)row * a.stride_o;
    }
    uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int col = c * 8 + e * 2;
            const float v0 = __uint_as_float(o[col >> 5][col & 31]) * inv_l;
            const float v1 = __uint_as_float(o[(col + 1) >> 5][(col + 1) & 31]) * inv_l;
#ifdef FMHA_O_ROUND_TRUNC
            pk[e] = pack_bf16_trunc(v0, v1);  // reference kernel's rounding
#else
            pk[e] = pack_bf16_rne(v0, v1);
#endif
        }
        dst[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    if (a.lse != nullptr) {
        long long idx;
        if constexpr (kVarlen) {
            idx = (long long)w.h * a.total_q + w.off_q + row;
        } else {
            idx = ((long long)w.b * a.nhead_q + w.h) * a.seqlen_q + row;
        }
        a.lse[idx] = lse;
    }
}

// Persistent CTA: loops over the work items work_index(k), k = 0, 1, ...
// Every role walks the same item sequence; the pipeline runs on as one flat
// stream of KV steps across query tiles (step counter g), so the first S of
// the next tile is computed while the softmax finishes the current one, and
// the next tile's Q is loaded (double buffer) while the current one runs.
template <bool kCausal, bool kVarlen>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
fmha_fwd_d64_sm100_kernel(const __grid_constant__ KernelArgs a) {
    extern __shared__ uint8_t smem_raw[];
    SharedStorage& sm = *reinterpret_cast<SharedStorage*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    volatile int* abort_flag = &sm.abort_flag;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&sm.bar_qfull[b]), 1);
            mbar_init(smem_u32(&sm.bar_qempty[b]), 1);
        }
        mbar_init(smem_u32(&sm.bar_s), 1);
        mbar_init(smem_u32(&sm.bar_sfree), 128);
        mbar_init(smem_u32(&sm.bar_p), 128);
        mbar_init(smem_u32(&sm.bar_pv), 1);
        mbar_init(smem_u32(&sm.bar_ofree), 128);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&sm.bar_full[s]), 1);
            mbar_init(smem_u32(&sm.bar_empty[s]), 1);
        }
        mbar_init(smem_u32(&sm.bar_drain), 1);
        sm.abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(smem_u32(&sm.tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    // Next item of this CTA with at least one KV tile, from round *k on.
    auto next_tile = [&](int& k, TileWork& w) -> bool {
        for (;; ++k) {
            const int x = work_index(a, k);
            if (x == -1) return false;
            if (x >= 0 && decode_work<kCausal, kVarlen>(a, x, w) && w.n > 0) {
                ++k;
                return true;
            }
        }
    };

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
            int q_issued = 0;  // Q loads issued (tile count)
            int issued = 0;    // K/V loads issued into the ring
            bool ok = true;
            auto issue_q = [&](const TileWork& w) -> bool {
                const int b = q_issued & 1;
                if (q_issued >= 2 &&
                    !wait_phase(smem_u32(&sm.bar_qempty[b]), ((q_issued - 2) >> 1) & 1,
                                abort_flag, a, kErrTimeoutLoad))
                    return false;
                const uint32_t bar = smem_u32(&sm.bar_qfull[b]);
                mbar_arrive_expect_tx(bar, kTileBytes);
                tma_load_rows<kVarlen>(smem_u32(sm.q[b]), &a.tm_q, bar, w.off_q + w.row0, w.h,
                                       kVarlen ? 0 : w.b, pol_q);
                ++q_issued;
                return true;
            };
            int k = 0;
            TileWork cur, nxt;
            bool have_cur = next_tile(k, cur);
            if (have_cur) ok = issue_q(cur);
            int gstep = 0;  // flat KV step counter (for the stall test hook)
            while (have_cur && ok) {
                const bool have_nxt = next_tile(k, nxt);
                for (int j = 0; j < cur.n && ok; ++j, ++gstep) {
                    for (int kv = 0; kv < 2; ++kv) {
                        const int idx = issued;
                        const int slot = idx % kStages;
                        const uint32_t use = idx / kStages;
                        if (!wait_phase(smem_u32(&sm.bar_empty[slot]), (use & 1) ^ 1, abort_flag,
                                        a, kErrTimeoutLoad)) {
                            ok = false;
                            break;
                        }
                        if (a.stall_inject && gstep == 0 && kv == 1) {
                            // Test hook: never deliver V_0, so the MMA warp's wait
                            // runs out and the abort path is exercised without
                            // any fault.
                            ok = false;
                            break;
                        }
                        const uint32_t bar = smem_u32(&sm.bar_full[slot]);
                        mbar_arrive_expect_tx(bar, kTileBytes);
                        tma_load_rows<kVarlen>(smem_u32(sm.kv[slot]), kv ? &a.tm_v : &a.tm_k,
                                               bar, cur.off_k + (cur.j0 + j) * kBlockN, cur.kvh,
                                               kVarlen ? 0 : cur.b, pol_kv);
                        issued = idx + 1;
                    }
                    // The next tile's Q goes out once this tile's first K/V is
                    // on its way.
                    if (ok && j == 0 && have_nxt) ok = issue_q(nxt);
                }
                cur = nxt;
                have_cur = have_nxt;
            }
            if (!ok || *abort_flag) {
                // Let every copy this warp started land before the CTA exits.
                for (int t = max(0, q_issued - 2); t < q_issued; ++t)
                    drain_phase(smem_u32(&sm.bar_qfull[t & 1]), (t >> 1) & 1, a);
                for (int idx = max(0, issued - kStages); idx < issued; ++idx)
                    drain_phase(smem_u32(&sm.bar_full[idx % kStages]), (idx / kStages) & 1, a);
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
        // S = Q K^T : M=128, N=128, K=64 as 4 x K16, 32 bytes (descriptor +2)
        // apart inside the 128-byte swizzled rows.
        auto issue_s = [&](int qb, int slot) {
            const uint64_t da = dq0 + (uint64_t)(qb * (kTileBytes >> 4));
            const uint64_t db = dk0 + (uint64_t)(slot * (kTileBytes >> 4));
            const uint32_t d = tmem + kColS;
            if (leader) {
                mma_ss(d, da, db, idesc_qk, 0u);
                mma_ss(d, da + 2, db + 2, idesc_qk, 1u);
                mma_ss(d, da + 4, db + 4, idesc_qk, 1u);
                mma_ss(d, da + 6, db + 6, idesc_qk, 1u);
            }
        };
        // O += P V : M=128, N=64, K=128 as 8 x K16.  P (bf16x2) is the TMEM A
        // operand; V is MN-major in shared memory, 16 keys = two 8-row
        // swizzle atoms = 2048 bytes (descriptor +128) per step.
        auto issue_pv = [&](int slot, bool accumulate) {
            const uint64_t db = dv0 + (uint64_t)(slot * (kTileBytes >> 4));
            const uint32_t d = tmem + kColO;
            const uint32_t pa = tmem + kColP;
            if (leader) {
                mma_ts(d, pa, db, idesc_pv, accumulate ? 1u : 0u);
#pragma unroll
                for (int kk = 1; kk < kBlockN / 16; ++kk)
                    mma_ts(d, pa + kk * 8, db + (uint64_t)(kk * 128), idesc_pv, 1u);
            }
        };
        // O += P(g) V(g) of flat step g; `first` starts a tile (O overwritten,
        // after the previous tile's O was read out), tile = its tile count.
        auto step_pv = [&](int g, bool first, int tile) -> bool {
            const int v_idx = 2 * g + 1;
            if (!wait_all(&sm.bar_full[slot_of(v_idx)], full_parity(v_idx))) return false;
            if (!wait_all(&sm.bar_p, g & 1)) return false;
            if (first && tile > 0 && !wait_all(&sm.bar_ofree, (tile - 1) & 1)) return false;
            tc_fence_after();
            issue_pv(slot_of(v_idx), !first);
            commit(&sm.bar_pv);
            commit(&sm.bar_empty[slot_of(v_idx)]);
            return true;
        };

        int k = 0;
        int g = 0;      // flat KV step counter
        int tile = 0;   // tiles with work seen by this CTA
        int pend_g = -1, pend_tile = 0;
        bool pend_first = false;
        TileWork w;
        while (ok && next_tile(k, w)) {
            const int qb = tile & 1;
            ok = wait_all(&sm.bar_qfull[qb], (tile >> 1) & 1);
            for (int j = 0; j < w.n && ok; ++j, ++g) {
                // S(g) as soon as the softmax has read S(g-1) and K landed ...
                const int k_idx = 2 * g;
                ok = wait_all(&sm.bar_full[slot_of(k_idx)], full_parity(k_idx));
                if (ok && g > 0) ok = wait_all(&sm.bar_sfree, (g - 1) & 1);
                if (!ok) break;
                tc_fence_after();
                issue_s(qb, slot_of(k_idx));
                commit(&sm.bar_s);
                commit(&sm.bar_empty[slot_of(k_idx)]);
                if (j == w.n - 1) commit(&sm.bar_qempty[qb]);
                // ... then O += P(g-1) V(g-1) once P(g-1) is written.
                if (pend_g >= 0) ok = step_pv(pend_g, pend_first, pend_tile);
                pend_g = g;
                pend_first = (j == 0);
                pend_tile = tile;
            }
            ++tile;
        }
        if (ok && pend_g >= 0) ok = step_pv(pend_g, pend_first, pend_tile);
        // All MMAs this warp issued must finish before TMEM is freed.
        commit(&sm.bar_drain);
        drain_phase(smem_u32(&sm.bar_drain), 0, a);
        __syncwarp();
    }
    } else {
        regs_inc<kRegsSoftmax>();
        // ------------------------------------------------------ softmax group
        const int t = threadIdx.x;  // row inside the tile == TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        const uint32_t tS = tmem + lane_base + kColS;
        const uint32_t tO = tmem + lane_base + kColO;
        const uint32_t tP = tmem + lane_base + kColP;
        const float scale = a.scale;
        bool ok = true;
        int g = 0;      // flat KV step counter
        // The tile description is parked in shared memory (one copy per warp)
        // while the KV loop runs, so its fields hold no registers there; the
        // loop itself needs only the scalars below.
        TileWork* wsave = &sm.work[warp];
        for (int k = 0; ok; ++k) {
            const int x = work_index(a, k);
            if (x == -1) break;
            int n, k0, tile_lim, key_lim;
            {
                TileWork w;
                if (x < 0 || !decode_work<kCausal, kVarlen>(a, x, w)) continue;
                n = w.n;
                k0 = w.j0 * kBlockN;
                const int shift = w.seqlen_k - w.seqlen_q;
                // Keys visible to this row: [0, key_lim); a KV tile needs the
                // mask once it reaches past the smallest limit of its rows.
                key_lim = kCausal ? min(w.seqlen_k, w.row0 + t + shift + 1) : w.seqlen_k;
                tile_lim = kCausal ? min(w.seqlen_k, w.row0 + shift + 1) : w.seqlen_k;
                if (lane == 0) *wsave = w;
                __syncwarp();
            }

            float m_run = -INFINITY;  // un-scaled running max used as exp2 reference
            float l_run = 0.0f;       // running sum of un-normalised P

            for (int j = 0; j < n; ++j, ++g) {
                bool got = wait_phase(smem_u32(&sm.bar_s), g & 1, abort_flag, a,
                                      kErrTimeoutSoftmax);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t r[4][32];
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, r[c]);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 4; ++c) reg_fence(r[c]);
                // S now lives in registers: the MMA warp may overwrite it with
                // S(g+1) while this group computes P(g).
                tc_fence_before();
                mbar_arrive(smem_u32(&sm.bar_sfree));

                const bool need_mask = k0 + kBlockN > tile_lim;
                if (need_mask) {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (k0 + c * 32 + e >= key_lim) r[c][e] = __float_as_uint(-INFINITY);
                }
                k0 += kBlockN;
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
                const float row_max = fmax3(fmax3(mx[0], mx[1], mx[2]),
                                            fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
                const float m_new = fmaxf(m_run, row_max);
                const bool upd = (m_new - m_run) * scale > kRescaleThreshold;
                float alpha = 1.0f;
                if (upd) {
                    alpha = ex2_approx((m_run - m_new) * scale);
                    m_run = m_new;
                }
                const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
                const float neg_ms = kPLog2Bias - m_use * scale;
                const float2 scale2 = make_float2(scale, scale);
                const float2 neg2 = make_float2(neg_ms, neg_ms);
                float2 sum[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) sum[q] = make_float2(0.0f, 0.0f);
                uint32_t p[2][32];
                // P = exp2(S*scale - m*scale).  On tiles without masking a
                // fixed share of the pairs (kExpPolyPairs of every 16) runs the
                // polynomial exp2 on the FMA/ALU pipes, relieving MUFU; masked
                // tiles (which may hold -inf) use MUFU ex2 only.
                auto exp_tile = [&](auto poly_tag) {
                    constexpr bool kPoly = decltype(poly_tag)::value;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            const int pr = e >> 1;  // pair index in the chunk
                            const float2 xx = ffma2(make_float2(__uint_as_float(r[c][e]),
                                                                __uint_as_float(r[c][e + 1])),
                                                    scale2, neg2);
                            float2 pp;
                            if (kPoly && ((pr + 1) * kExpPolyPairs / 16 > pr * kExpPolyPairs / 16))
                                pp = exp2_poly2(xx);
                            else
                                pp = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
                            sum[pr & 3] = fadd2(sum[pr & 3], pp);
                            p[c >> 1][(c & 1) * 16 + pr] = pack_bf16_trunc(pp.x, pp.y);
                        }
                };
                if (need_mask) exp_tile(std::false_type{});
                else exp_tile(std::true_type{});
                const float2 s01 = fadd2(fadd2(sum[0], sum[1]), fadd2(sum[2], sum[3]));
                l_run = fmaf(l_run, alpha, s01.x + s01.y);

                if (g > 0) {
                    // P(g-1) must be consumed (and O settled) before P(g) and
                    // the O rescale are written.
                    got = wait_phase(smem_u32(&sm.bar_pv), (g - 1) & 1, abort_flag, a,
                                     kErrTimeoutSoftmax);
                    if (!__all_sync(0xffffffffu, got)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
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
                            const float2 v2 = fmul2(
                                make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), a2);
                            o[e] = __float_as_uint(v2.x);
                            o[e + 1] = __float_as_uint(v2.y);
                        }
                        tmem_st32(tO + c * 32, o);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(smem_u32(&sm.bar_p));
            }
            if (!ok) break;

            // ---------------------------------------------------- epilogue
            uint32_t o[2][32];
            if (n == 0) {
#pragma unroll
                for (int c = 0; c < 32; ++c) o[0][c] = o[1][c] = 0u;
            } else {
                // The tile's last P V is done: read O out, then hand the
                // accumulator to the next tile's first P V.
                bool got = wait_phase(smem_u32(&sm.bar_pv), (g - 1) & 1, abort_flag, a,
                                      kErrTimeoutSoftmax);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                tmem_ld32(tO, o[0]);
                tmem_ld32(tO + 32, o[1]);
                tmem_wait_ld();
                reg_fence(o[0]);
                reg_fence(o[1]);
                tc_fence_before();
                mbar_arrive(smem_u32(&sm.bar_ofree));
            }
            __syncwarp();
            const TileWork w = *wsave;
            __syncwarp();  // every lane has its copy before the next tile's write
            store_row<kVarlen>(a, w, t, o, n > 0, m_run, l_run);
        }
    }

    // ---------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Split-KV merge of one query row: partial slots [slot0, slot0 + nparts) of
// query block mblk of (batch, head) hb; LSE = log(sum_s exp(lse_s)),
// O = sum_s exp(lse_s - LSE) * O_s, rounded to bf16 like the main epilogue;
// the same LSE merge the reference's base-2 epilogue formula implies
// (src/fused/op_epilog.hpp:92-98).
template <bool kVarlen>
__device__ __forceinline__ void merge_row(const KernelArgs& a, int hb, int mblk, int slot0,
                                          int nparts, int r) {
    // Malformed list entries are skipped before any address is formed.
    if (hb < 0 || hb >= a.num_hb || mblk < 0 || mblk >= a.m_blocks) return;
    const int h = hb % a.nhead_q, b = hb / a.nhead_q;
    int seqlen_q = a.seqlen_q, off_q = 0;
    if constexpr (kVarlen) {
        off_q = a.seqstart_q[b];
        seqlen_q = a.seqstart_q[b + 1] - off_q;
        if (off_q < 0 || seqlen_q < 0 || off_q + seqlen_q > a.total_q) return;
    }
    const int row = mblk * kBlockM + r;
    if (row >= seqlen_q) return;
    float mx = -INFINITY;
    for (int s = 0; s < nparts; ++s)
        mx = fmaxf(mx, a.part_lse[(size_t)(slot0 + s) * kBlockM + r]);
    float acc[kHeadDim];
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) acc[d] = 0.0f;
    float wsum = 0.0f;
    if (mx != -INFINITY) {
        for (int s = 0; s < nparts; ++s) {
            const size_t prow = (size_t)(slot0 + s) * kBlockM + r;
            const float l = a.part_lse[prow];
            if (l == -INFINITY) continue;
            const float wgt = __expf(l - mx);
            wsum += wgt;
            const float4* src = reinterpret_cast<const float4*>(a.part_o + prow * kHeadDim);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const float4 v = src[c];
                acc[4 * c] += wgt * v.x;
                acc[4 * c + 1] += wgt * v.y;
                acc[4 * c + 2] += wgt * v.z;
                acc[4 * c + 3] += wgt * v.w;
            }
        }
    }
    const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
    uint16_t* orow;
    if constexpr (kVarlen) {
        orow = a.o + (long long)h * a.nhead_stride_o + (long long)(off_q + row) * a.stride_o;
    } else {
        orow = a.o + (long long)b * a.batch_stride_o + (long long)h * a.nhead_stride_o +
               (long long)row * a.stride_o;
    }
    uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
#ifdef FMHA_O_ROUND_TRUNC
            pk[e] = pack_bf16_trunc(acc[c * 8 + 2 * e] * inv, acc[c * 8 + 2 * e + 1] * inv);
#else
            pk[e] = pack_bf16_rne(acc[c * 8 + 2 * e] * inv, acc[c * 8 + 2 * e + 1] * inv);
#endif
        }
        dst[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    if (a.lse != nullptr) {
        const float lse = wsum > 0.0f ? mx + __logf(wsum) : -INFINITY;
        const long long idx = kVarlen ? (long long)h * a.total_q + off_q + row
                                      : ((long long)b * a.nhead_q + h) * a.seqlen_q + row;
        a.lse[idx] = lse;
    }
}

// Uniform split-KV combine: block g merges slots [g*S, g*S + S) of tiles[g].
template <bool kVarlen>
__global__ void __launch_bounds__(128)
fmha_fwd_d64_splitkv_combine(const __grid_constant__ KernelArgs a, int nblocks) {
    const int item_block = blockIdx.x;
    if (item_block >= nblocks) return;
    merge_row<kVarlen>(a, a.tiles[2 * item_block], a.tiles[2 * item_block + 1],
                       item_block * a.num_splits, a.num_splits, threadIdx.x);
}

// Work-item combine: block x merges the run of consecutive partial items of
// one query block that starts at item x (other blocks return at once).  The
// run length is found with one parallel probe per thread (128 items per
// pass), not a chain of dependent loads.
template <bool kVarlen>
__global__ void __launch_bounds__(128)
fmha_fwd_d64_items_combine(const __grid_constant__ KernelArgs a, int n_items) {
    __shared__ int run_end;
    const int x = blockIdx.x;
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
    for (int base = x + 1;; base += 128) {
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
        if (e < base + 128 || base + 128 >= n_items) {
            n = min(e, n_items) - x;
            break;
        }
    }
    merge_row<kVarlen>(a, it.x, it.y, x, n, threadIdx.x);
}

// ====================================================================== host

struct DeviceContext {
    bool ready = false;
    int num_sms = 0;
    int* err_word = nullptr;
};

std::mutex g_mutex;
std::vector<DeviceContext> g_devices;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
unsigned long long g_wait_limit_ns = 2000000000ull;
int g_stall_inject = 0;
int g_max_ctas = 0;  // 0: kCtasPerSm per SM (persistent); < 0: one CTA per item

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

// Per device, once (device current): check it is an sm_100 part, read its SM
// count and set the kernels' shared-memory attributes.  Allocates nothing.
int prepare_device(int dev, int* num_sms) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return FMHA_ERR_DEVICE;
    if (prop.major != 10 || prop.minor != 0) return FMHA_ERR_DEVICE;
    *num_sms = prop.multiProcessorCount;
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
        if ((st = prepare_device(dev, &ctx.num_sms)) != FMHA_OK) return st;
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

// Persistent grid: at most kCtasPerSm CTAs per SM (or the caller's limit),
// never more CTAs than work items.
unsigned grid_for(int n_work, int num_sms) {
    long long cap = (long long)kCtasPerSm * num_sms;
    if (g_max_ctas > 0) cap = std::min<long long>(cap, g_max_ctas);
    if (g_max_ctas < 0) cap = n_work;
    return (unsigned)std::max(1ll, std::min<long long>(cap, n_work));
}

int launch_main(const KernelArgs& a, bool causal, bool varlen, unsigned grid,
                cudaStream_t stream) {
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

    a.n_work = a.m_blocks * a.num_hb;
    a.tiles = tiles;
    if (tiles != nullptr) {
        if (ntiles == 0) return FMHA_OK;
        a.n_work = ntiles;
        if (num_splits > 1) {
            a.num_splits = num_splits;
            a.part_o = workspace;
            a.part_lse = workspace + (size_t)ntiles * num_splits * kBlockM * kHeadDim;
            a.n_work = ntiles * num_splits;
        }
    }
    if (items != nullptr) {
        if (n_items == 0) return FMHA_OK;
        a.items = items;
        a.part_o = workspace;
        a.part_lse = workspace + (size_t)n_items * kBlockM * kHeadDim;
        a.n_work = n_items;
    }
    if ((st = launch_main(a, causal, varlen, grid_for(a.n_work, ctx->num_sms), stream)) !=
        FMHA_OK)
        return st;
    if (items != nullptr) {
        dim3 cgrid((unsigned)n_items, 1, 1);
        if (varlen) fmha_fwd_d64_items_combine<true><<<cgrid, 128, 0, stream>>>(a, n_items);
        else fmha_fwd_d64_items_combine<false><<<cgrid, 128, 0, stream>>>(a, n_items);
    } else if (a.num_splits > 1) {
        dim3 cgrid((unsigned)ntiles, 1, 1);
        if (varlen) fmha_fwd_d64_splitkv_combine<true><<<cgrid, 128, 0, stream>>>(a, ntiles);
        else fmha_fwd_d64_splitkv_combine<false><<<cgrid, 128, 0, stream>>>(a, ntiles);
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
    int num_sms = 0;
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
        if ((st = prepare_device(dev, &d.num_sms)) != FMHA_OK) return st;
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
    KernelArgs a;
    bool empty = false;
    int st = prepare_args(p, batch, varlen, total_q, total_k, a, &empty);
    if (st != FMHA_OK) return st;
    // The list is on the host, so every entry is checked before anything is
    // queued: a (batch, head) index or query block outside the problem is an
    // argument error, not a silent skip.
    const long long num_hb = (long long)p->nhead_q * batch;
    const int m_blocks = (p->seqlen_q + kBlockM - 1) / kBlockM;
    for (int i = 0; i < ntiles; ++i) {
        const int32_t hb = host_tiles[2 * i], m = host_tiles[2 * i + 1];
        if (hb < 0 || hb >= num_hb || m < 0 || m >= m_blocks) return FMHA_ERR_ARG;
    }
    if (ntiles == 0 || empty) return FMHA_OK;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_DEVICE;
    NoAllocDevice* d = nullptr;
    if ((st = noalloc_setup(dev, &d)) != FMHA_OK) return st;
    int32_t* scratch = d->scratch;
    a.err_word = scratch;  // header word 0
    a.stall_inject = 0;
    a.tiles = scratch + kNoAllocHeaderInts;
    a.n_work = ntiles;

    // The array keeps the previous call's contents: clear the error word and
    // stage this call's work list, in stream order before the kernel.
    if (cudaMemsetAsync(scratch, 0, sizeof(int32_t), stream) != cudaSuccess) return FMHA_ERR_LAUNCH;
    if (cudaMemcpyAsync(scratch + kNoAllocHeaderInts, host_tiles,
                        sizeof(int32_t) * 2 * (size_t)ntiles, cudaMemcpyHostToDevice,
                        stream) != cudaSuccess)
        return FMHA_ERR_LAUNCH;
    return launch_main(a, causal, varlen, grid_for(ntiles, d->num_sms), stream);
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

void fmha_fwd_d64_set_max_ctas(int max_ctas) {
    std::lock_guard<std::mutex> lock(g_mutex);
    g_max_ctas = max_ctas > 0 ? max_ctas : (max_ctas < 0 ? -1 : 0);
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
