// TEST INFRASTRUCTURE ONLY.  extern "C" entry points over the reference's own
// CPU oracle (src/runner/cpu_ref.cpp) and input generator
// (src/runner/buffers.cpp: FmhaBuffers::fill_random), both compiled
// unmodified from the reference tree by oracle/build.py into
// oracle/_ref/libfmha_ref.so.  Used by tests/ to pin oracle/fmha_oracle.c and
// by bench.py's reference (CPU baseline) arm.
//
// Data layouts are the reference oracle's: dense BHSD [B,H,S,64], varlen
// [H,total,64] (cpu_ref.cpp:92-100).
#include <cstdint>
#include <cstring>
#include <vector>

#include "buffers.hpp"
#include "cpu_ref.hpp"
#include "fmha_params.hpp"

namespace {
// Same derivations as the reference test helper make_params
// (tests/test_params.hpp:31-61), head_dim fixed at 64.
FmhaParams make(int batch, int q_heads, int kv_heads, int seq_len, int kv_seq_len, int mask,
                const int* varlen, int nvarlen) {
    FmhaParams p;
    p.batch = batch;
    p.q_heads = q_heads;
    p.kv_heads = kv_heads ? kv_heads : q_heads;
    p.gqa = p.q_heads / p.kv_heads;
    p.seq_len = seq_len;
    p.kv_seq_len = kv_seq_len;
    p.head_dim = 64;
    p.hdim_padded = 64;
    p.mask = mask;
    p.lse = 0;
    if (varlen && nvarlen > 0) {
        p.varlen_seqs.assign(varlen, varlen + nvarlen);
        p.batch = nvarlen;
        int mx = 0;
        for (int s : p.varlen_seqs) mx = s > mx ? s : mx;
        p.seq_len = mx;
        if (p.kv_seq_len == 0) p.kv_seq_len = mx;
    }
    if (p.kv_seq_len == 0) p.kv_seq_len = p.seq_len;
    return p;
}
}  // namespace

extern "C" {

struct RefVerdict {
    int pass;
    double max_abs, max_rel, min_cos, mean_cos;
    unsigned long long mismatch, nonfinite, total_elems, cos_fail, cos_rows;
    int worst_b, worst_h, worst_i, worst_d;
    float worst_ref, worst_kern;
};

// Element counts the reference allocates for Q, K(=V) and O.
void ref_sizes(int batch, int q_heads, int kv_heads, int seq_len, int kv_seq_len,
               const int* varlen, int nvarlen, unsigned long long out[3]) {
    FmhaParams p = make(batch, q_heads, kv_heads, seq_len, kv_seq_len, 0, varlen, nvarlen);
    FmhaBuffers bufs(p);
    out[0] = bufs.sz_Q;
    out[1] = bufs.sz_K;
    out[2] = bufs.sz_O;
}

// Reference input generator (buffers.cpp:99-127) into caller buffers.
void ref_fill_random(int batch, int q_heads, int kv_heads, int seq_len, int kv_seq_len,
                     const int* varlen, int nvarlen, unsigned seed, uint16_t* q, uint16_t* k,
                     uint16_t* v) {
    FmhaParams p = make(batch, q_heads, kv_heads, seq_len, kv_seq_len, 0, varlen, nvarlen);
    FmhaBuffers bufs(p);
    bufs.fill_random(seed);
    std::memcpy(q, bufs.h_Q.data(), bufs.sz_Q * 2);
    std::memcpy(k, bufs.h_K.data(), bufs.sz_K * 2);
    std::memcpy(v, bufs.h_V.data(), bufs.sz_V * 2);
}

// Reference verdict (cpu_ref_verify, cpu_ref.cpp:14-311) of kernel output `o`.
int ref_verify(int batch, int q_heads, int kv_heads, int seq_len, int kv_seq_len, int mask,
               const int* varlen, int nvarlen, const uint16_t* q, const uint16_t* k,
               const uint16_t* v, const uint16_t* o, RefVerdict* out) {
    FmhaParams p = make(batch, q_heads, kv_heads, seq_len, kv_seq_len, mask, varlen, nvarlen);
    FmhaBuffers bufs(p);
    std::memcpy(bufs.h_Q.data(), q, bufs.sz_Q * 2);
    std::memcpy(bufs.h_K.data(), k, bufs.sz_K * 2);
    std::memcpy(bufs.h_V.data(), v, bufs.sz_V * 2);
    bufs.h_O.assign(o, o + bufs.sz_O);
    CpuRefResult r = cpu_ref_verify(p, bufs);
    out->pass = r.pass ? 1 : 0;
    out->max_abs = r.max_abs;
    out->max_rel = r.max_rel;
    out->min_cos = r.min_cos;
    out->mean_cos = r.mean_cos;
    out->mismatch = r.mismatch;
    out->nonfinite = r.nonfinite;
    out->total_elems = r.total_elems;
    out->cos_fail = r.cos_fail;
    out->cos_rows = r.cos_rows;
    out->worst_b = r.worst_b;
    out->worst_h = r.worst_h;
    out->worst_i = r.worst_i;
    out->worst_d = r.worst_d;
    out->worst_ref = r.worst_ref;
    out->worst_kern = r.worst_kern;
    return r.pass ? 1 : 0;
}

}  // extern "C"
