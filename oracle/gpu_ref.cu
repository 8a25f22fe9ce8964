// gpu_ref.cu -- TEST INFRASTRUCTURE ONLY: a plain-CUDA fp32 device oracle of
// the D64 attention forward, for parity checks at sizes where the CPU oracle
// would take minutes (full BASELINE configurations).  Nothing in the product
// library links or calls it; tests/, __graft_entry__.smoke() and bench.py's
// CPU leg are its only users.
//
// Restates the reference's naive GPU reference, src/runner/gpu_ref.cpp:12-126
// (one thread per query row, three passes over the keys):
//   pass 1  m   = max_j s_j,            s_j = (q . k_j) / sqrt(64), masked -inf
//   pass 2  l   = sum_j exp(s_j - m)
//   pass 3  O   = sum_j bf16_trunc(exp(s_j - m) / l) * v_j      (:89-111)
//   LSE = log(l) + m, -inf when l == 0                           (:116-125)
// with the reference's bottom-right causal rule (mask j > i + (Sk - Sq), :66)
// and varlen offsets from seqstart (:35-46).  The dot product runs in d
// order and the key loops in key order, as there.  Differences from the
// reference's code, none affecting a value: K/V rows are staged through
// shared memory 32 keys at a time for the 128 rows of a block, O and LSE are
// written as fp32 (so callers compare against the unrounded result), and the
// LSE layout is explicit ([B,H,Sq] dense, [H,total_q] varlen).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

namespace {

constexpr int kD = 64;
constexpr int kRows = 128;   // query rows per block (all of one batch, head)
constexpr int kChunk = 32;   // keys staged per pass step

struct GpuRefArgs {
    const uint16_t* q;
    const uint16_t* k;
    const uint16_t* v;
    float* o;      // fp32, addressed with the o strides below
    float* lse;    // optional
    long long sq_row, sq_head, sq_batch;
    long long sk_row, sk_head, sk_batch;
    long long sv_row, sv_head, sv_batch;
    long long so_row, so_head, so_batch;
    int batch, nhead_q, nhead_k, seqlen_q, seqlen_k, causal;
    const int32_t* seqstart_q;  // varlen when non-null
    const int32_t* seqstart_k;
    int total_q;
    float scale;   // 1/sqrt(64)
};

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ float bf16_trunc(float x) {
    return __uint_as_float(__float_as_uint(x) & 0xffff0000u);
}

__global__ void __launch_bounds__(kRows) gpu_ref_kernel(GpuRefArgs a) {
    __shared__ float ks[kChunk][kD + 1];
    __shared__ float vs[kChunk][kD + 1];
    const int mblocks = (a.seqlen_q + kRows - 1) / kRows;
    const int blk = blockIdx.x;
    const int mb = blk % mblocks;
    const int h = (blk / mblocks) % a.nhead_q;
    const int b = blk / (mblocks * a.nhead_q);
    const int kvh = h / (a.nhead_q / a.nhead_k);
    int sq = a.seqlen_q, sk = a.seqlen_k, oq = 0, ok = 0;
    if (a.seqstart_q) {
        oq = a.seqstart_q[b];
        ok = a.seqstart_k[b];
        sq = a.seqstart_q[b + 1] - oq;
        sk = a.seqstart_k[b + 1] - ok;
    }
    const int i = mb * kRows + threadIdx.x;       // query row of this thread
    const int row0 = mb * kRows;
    if (row0 >= sq) return;                       // whole block past the sequence
    const bool active = i < sq;
    const int shift = sk - sq;
    // Keys any row of the block may see (the block stages this range).
    int kend = sk;
    if (a.causal) kend = min(sk, min(row0 + kRows - 1, sq - 1) + shift + 1);
    const int my_lim = a.causal ? min(sk, i + shift + 1) : sk;

    const long long qbase = (a.seqstart_q ? 0 : (long long)b * a.sq_batch) +
                            (long long)h * a.sq_head + (long long)(oq + (active ? i : 0)) * a.sq_row;
    const long long kbase = (a.seqstart_q ? 0 : (long long)b * a.sk_batch) + (long long)kvh * a.sk_head +
                            (long long)ok * a.sk_row;
    const long long vbase = (a.seqstart_q ? 0 : (long long)b * a.sv_batch) + (long long)kvh * a.sv_head +
                            (long long)ok * a.sv_row;
    float q[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) q[d] = active ? bf16f(a.q[qbase + d]) : 0.0f;

    auto stage = [&](int j0, bool with_v) {
        __syncthreads();
        for (int e = threadIdx.x; e < kChunk * kD; e += kRows) {
            const int jj = e / kD, d = e % kD;
            const int j = j0 + jj;
            ks[jj][d] = j < kend ? bf16f(a.k[kbase + (long long)j * a.sk_row + d]) : 0.0f;
            if (with_v) vs[jj][d] = j < kend ? bf16f(a.v[vbase + (long long)j * a.sv_row + d]) : 0.0f;
        }
        __syncthreads();
    };
    auto score = [&](int jj) {
        float s = 0.0f;
#pragma unroll
        for (int d = 0; d < kD; ++d) s = __fadd_rn(s, __fmul_rn(q[d], ks[jj][d]));
        return __fmul_rn(s, a.scale);
    };

    // Pass 1: row max.
    float m = -INFINITY;
    for (int j0 = 0; j0 < kend; j0 += kChunk) {
        stage(j0, false);
        for (int jj = 0; jj < kChunk && j0 + jj < kend; ++jj) {
            const float s = (j0 + jj < my_lim) ? score(jj) : -INFINITY;
            if (s > m) m = s;
        }
    }
    // Pass 2: denominator.
    float l = 0.0f;
    for (int j0 = 0; j0 < kend; j0 += kChunk) {
        stage(j0, false);
        for (int jj = 0; jj < kChunk && j0 + jj < kend; ++jj) {
            if (j0 + jj < my_lim) l += expf(score(jj) - m);
        }
    }
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    // Pass 3: O = sum bf16_trunc(p / l) * v.
    float acc[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) acc[d] = 0.0f;
    for (int j0 = 0; j0 < kend; j0 += kChunk) {
        stage(j0, true);
        for (int jj = 0; jj < kChunk && j0 + jj < kend; ++jj) {
            if (j0 + jj >= my_lim) continue;
            const float p = bf16_trunc(expf(score(jj) - m) * inv);
#pragma unroll
            for (int d = 0; d < kD; ++d) acc[d] = __fadd_rn(acc[d], __fmul_rn(p, vs[jj][d]));
        }
    }
    if (!active) return;
    const long long obase = (a.seqstart_q ? 0 : (long long)b * a.so_batch) + (long long)h * a.so_head +
                            (long long)(oq + i) * a.so_row;
#pragma unroll
    for (int d = 0; d < kD; ++d) a.o[obase + d] = acc[d];
    if (a.lse) {
        const float lse = l > 0.0f ? logf(l) + m : -INFINITY;
        const long long li = a.seqstart_q ? (long long)h * a.total_q + oq + i
                                          : ((long long)b * a.nhead_q + h) * a.seqlen_q + i;
        a.lse[li] = lse;
    }
}

}  // namespace

extern "C" {

// Runs the oracle on device buffers (strides in elements; o/lse fp32).
// Returns 0 or the CUDA error code of the launch.
int gpu_ref_fmha_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, float* lse,
                     const long long* strides /* 12: q,k,v,o x (row, head, batch) */, int batch,
                     int nhead_q, int nhead_k, int seqlen_q, int seqlen_k, int causal,
                     const int32_t* seqstart_q, const int32_t* seqstart_k, int total_q,
                     float scale, cudaStream_t stream) {
    GpuRefArgs a;
    a.q = q; a.k = k; a.v = v; a.o = o; a.lse = lse;
    a.sq_row = strides[0]; a.sq_head = strides[1]; a.sq_batch = strides[2];
    a.sk_row = strides[3]; a.sk_head = strides[4]; a.sk_batch = strides[5];
    a.sv_row = strides[6]; a.sv_head = strides[7]; a.sv_batch = strides[8];
    a.so_row = strides[9]; a.so_head = strides[10]; a.so_batch = strides[11];
    a.batch = batch; a.nhead_q = nhead_q; a.nhead_k = nhead_k;
    a.seqlen_q = seqlen_q; a.seqlen_k = seqlen_k; a.causal = causal;
    a.seqstart_q = seqstart_q; a.seqstart_k = seqstart_k; a.total_q = total_q;
    a.scale = scale;
    if (seqlen_q <= 0 || batch <= 0) return 0;
    const long long blocks = (long long)batch * nhead_q * ((seqlen_q + kRows - 1) / kRows);
    gpu_ref_kernel<<<(unsigned)blocks, kRows, 0, stream>>>(a);
    return (int)cudaGetLastError();
}

}  // extern "C"
