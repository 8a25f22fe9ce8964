/*
 * fmha_oracle.c -- TEST INFRASTRUCTURE ONLY.  CPU restatement of the
 * reference's attention oracle, used as the parity checker by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg.  Never linked into
 * or called by the product library.
 *
 * Restated algorithms (poyenc/fmha_native):
 *   oracle_fill_random ... src/runner/buffers.cpp:99-127  (glibc srand/rand,
 *                          value ((rand()%1000)-500)/5000, truncated to bf16,
 *                          filled Q then K then V, row-major over all rows)
 *   oracle_fmha_fwd ...... src/runner/cpu_ref.cpp:86-144  (per query row:
 *                          S_j = (sum_d q_d*k_jd) * (1/sqrt(64)) accumulated
 *                          in fp32 in d order; bottom-right causal mask
 *                          j > i + (Sk-Sq) -> -inf (:120); max; expf(S-m);
 *                          sum; P = bf16_trunc(P * (1/sum)) (:138-142);
 *                          O_d = sum_j P_j * v_jd accumulated in j order)
 *                          plus LSE = logf(sum) + max, -inf when the row has
 *                          no visible key, from src/runner/gpu_ref.cpp:116-125
 *                          (the reference test's LSE oracle).
 *
 * Parity pin: tests/test_oracle.py checks this file against the reference's
 * own cpu_ref_verify / fill_random compiled from the reference sources into
 * oracle/_ref (see oracle/build.py), and against the committed golden
 * fixtures under tests/golden/.
 *
 * Build: gcc -O2 -fopenmp -shared -fPIC (no -ffast-math, no FMA contraction;
 * x86-64 baseline ISA so float arithmetic matches the reference's g++ build).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline uint16_t f2bf_trunc(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (uint16_t)(u >> 16);
}
static inline float bf2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Sequential glibc-rand fill of n elements (buffers.cpp:109-113 formula).
 * Call order matters: the reference fills Q, then K, then V after one srand. */
void oracle_srand(unsigned seed) { srand(seed); }
void oracle_fill_rand_bf16(uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float v = (float)((rand() % 1000) - 500) / 5000.0f;
        dst[i] = f2bf_trunc(v);
    }
}
void oracle_fill_random(unsigned seed, uint16_t* q, size_t nq, uint16_t* k, size_t nk,
                        uint16_t* v, size_t nv) {
    srand(seed);
    oracle_fill_rand_bf16(q, nq);
    oracle_fill_rand_bf16(k, nk);
    oracle_fill_rand_bf16(v, nv);
}

/* Problem description: element strides exactly as FmhaFwdParams. */
typedef struct OracleProblem {
    int batch, nhead_q, nhead_k, seqlen_q, seqlen_k, causal;
    long long stride_q, nhead_stride_q, batch_stride_q;
    long long stride_k, nhead_stride_k, batch_stride_k;
    long long stride_v, nhead_stride_v, batch_stride_v;
    /* output strides (elements) for o_ref (fp32) */
    long long stride_o, nhead_stride_o, batch_stride_o;
    /* varlen: host prefix sums (batch+1) or NULL */
    const int32_t* seqstart_q;
    const int32_t* seqstart_k;
    int total_q; /* varlen LSE head stride */
    /* compute rows with (i % row_step) == row_phase only (1/0 = all rows) */
    int row_step, row_phase;
} OracleProblem;

/* O_ref (fp32, written at o_ref with the output strides) and LSE (fp32,
 * dense [B,Hq,Sq] or varlen [Hq,total_q]; lse may be NULL).  Rows not
 * selected by row_step/row_phase are left untouched. */
void oracle_fmha_fwd(const OracleProblem* p, const uint16_t* q, const uint16_t* k,
                     const uint16_t* v, float* o_ref, float* lse) {
    const int D = 64;
    const float scalar = 1.0f / sqrtf(64.0f);
    const int ratio = p->nhead_q / p->nhead_k;
    const int step = p->row_step > 0 ? p->row_step : 1;
    int max_sk = p->seqlen_k;
    if (p->seqstart_k) {
        max_sk = 0;
        for (int b = 0; b < p->batch; ++b) {
            int s = p->seqstart_k[b + 1] - p->seqstart_k[b];
            if (s > max_sk) max_sk = s;
        }
    }

#pragma omp parallel
    {
        float* S = (float*)malloc(sizeof(float) * (size_t)(max_sk > 0 ? max_sk : 1));
        float* P = (float*)malloc(sizeof(float) * (size_t)(max_sk > 0 ? max_sk : 1));
        for (int b = 0; b < p->batch; ++b)
            for (int h = 0; h < p->nhead_q; ++h) {
                const int hk = h / ratio;
                int sq = p->seqlen_q, sk = p->seqlen_k, oq = 0, ok = 0;
                if (p->seqstart_q) {
                    oq = p->seqstart_q[b];
                    sq = p->seqstart_q[b + 1] - oq;
                    ok = p->seqstart_k[b];
                    sk = p->seqstart_k[b + 1] - ok;
                }
                /* rows are independent: spread them over threads (no barrier
                 * between (b,h) pairs) */
#pragma omp for schedule(dynamic, 4) nowait
                for (int i = 0; i < sq; ++i) {
                    if ((i % step) != p->row_phase) continue;
                    const uint16_t* qr;
                    const uint16_t* kb;
                    const uint16_t* vb;
                    float* orow;
                    if (p->seqstart_q) {
                        qr = q + h * p->nhead_stride_q + (long long)(oq + i) * p->stride_q;
                        kb = k + hk * p->nhead_stride_k + (long long)ok * p->stride_k;
                        vb = v + hk * p->nhead_stride_v + (long long)ok * p->stride_v;
                        orow = o_ref + h * p->nhead_stride_o + (long long)(oq + i) * p->stride_o;
                    } else {
                        qr = q + b * p->batch_stride_q + h * p->nhead_stride_q + (long long)i * p->stride_q;
                        kb = k + b * p->batch_stride_k + hk * p->nhead_stride_k;
                        vb = v + b * p->batch_stride_v + hk * p->nhead_stride_v;
                        orow = o_ref + b * p->batch_stride_o + h * p->nhead_stride_o + (long long)i * p->stride_o;
                    }
                    for (int j = 0; j < sk; ++j) {
                        float s = 0.0f;
                        const uint16_t* kr = kb + (long long)j * p->stride_k;
                        for (int d = 0; d < D; ++d) s += bf2f(qr[d]) * bf2f(kr[d]);
                        S[j] = s * scalar;
                        if (p->causal && j > i + (sk - sq)) S[j] = -INFINITY;
                    }
                    float m = sk > 0 ? S[0] : -INFINITY;
                    for (int j = 1; j < sk; ++j)
                        if (S[j] > m) m = S[j];
                    float sum = 0.0f;
                    if (m == -INFINITY) {
                        for (int j = 0; j < sk; ++j) P[j] = 0.0f;
                    } else {
                        for (int j = 0; j < sk; ++j) {
                            P[j] = (isinf(S[j]) && S[j] < 0) ? 0.0f : expf(S[j] - m);
                            sum += P[j];
                        }
                        const float inv = 1.0f / sum;
                        for (int j = 0; j < sk; ++j) P[j] = bf2f(f2bf_trunc(P[j] * inv));
                    }
                    for (int d = 0; d < D; ++d) {
                        float acc = 0.0f;
                        for (int j = 0; j < sk; ++j) acc += P[j] * bf2f(vb[(long long)j * p->stride_v + d]);
                        orow[d] = acc;
                    }
                    if (lse) {
                        long long li = p->seqstart_q
                                           ? (long long)h * p->total_q + oq + i
                                           : ((long long)b * p->nhead_q + h) * p->seqlen_q + i;
                        lse[li] = (sum > 0.0f) ? logf(sum) + m : -INFINITY;
                    }
                }
            }
        free(S);
        free(P);
    }
}
