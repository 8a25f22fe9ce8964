// bench_fmha_fwd -- timing CLI for the B200 D64 BF16 FMHA forward, with the
// reference's command line and output lines (src/bench_fmha_fwd.cpp:43-56,
// 231-233): -b -h --kv-heads -s -d --mask --lse --varlen-seqs --warmup --iters
// and "Avg: X ms" / "min=X ms" / "TFLOPS: X".  Inputs follow the reference
// generator (glibc srand(42), ((rand()%1000)-500)/5000 truncated to bf16,
// src/runner/buffers.cpp:99-127) in the reference layouts (BHSD dense,
// [H,total,D] varlen).  Varlen FLOPs count sum_b S_b^2 (the reference counts
// max_S^2 per sequence).
#include <cuda_runtime.h>
#include <getopt.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "fmha_fwd.h"

#define CUDA_CHECK(x)                                                                  \
    do {                                                                               \
        cudaError_t e_ = (x);                                                          \
        if (e_ != cudaSuccess) {                                                       \
            fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, \
                    __LINE__);                                                         \
            return 1;                                                                  \
        }                                                                              \
    } while (0)

static uint16_t f2bf_trunc(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (uint16_t)(u >> 16);
}

static void usage(const char* prog) {
    printf("Usage: %s [options]\n"
           "  -b  --batch N    Batch size [2]\n"
           "  -h  --heads N    Q head count [16]\n"
           "  --kv-heads N     KV head count [0 = q_heads]\n"
           "  -s  --seq N      Sequence length [4096]\n"
           "  -d  --hdim N     Head dimension [64] (only 64 is supported)\n"
           "  --mask N         Causal mask 0|1 [0]\n"
           "  --lse N          LSE output enable [0]\n"
           "  --varlen-seqs L  Per-batch seq lengths (comma-separated)\n"
           "  --warmup N       Warmup iterations [5]\n"
           "  --iters N        Benchmark iterations [20]\n",
           prog);
}

int main(int argc, char** argv) {
    int batch = 2, heads = 16, kv_heads = 0, seq = 4096, hdim = 64, mask = 0, lse = 0;
    int warmup = 5, iters = 20;
    std::vector<int> varlen;
    static struct option opts[] = {
        {"varlen-seqs", required_argument, 0, 6}, {"batch", required_argument, 0, 'b'},
        {"heads", required_argument, 0, 'h'},     {"kv-heads", required_argument, 0, 1},
        {"seq", required_argument, 0, 's'},       {"hdim", required_argument, 0, 'd'},
        {"mask", required_argument, 0, 'm'},      {"lse", required_argument, 0, 'l'},
        {"warmup", required_argument, 0, 'w'},    {"iters", required_argument, 0, 'i'},
        {"help", no_argument, 0, 0},              {0, 0, 0, 0}};
    int c, idx;
    while ((c = getopt_long(argc, argv, "b:h:s:d:m:l:w:i:", opts, &idx)) != -1) {
        switch (c) {
            case 6: {
                for (const char* p = optarg; *p;) {
                    varlen.push_back(atoi(p));
                    while (*p && *p != ',') ++p;
                    if (*p) ++p;
                }
                break;
            }
            case 'b': batch = atoi(optarg); break;
            case 'h': heads = atoi(optarg); break;
            case 1: kv_heads = atoi(optarg); break;
            case 's': seq = atoi(optarg); break;
            case 'd': hdim = atoi(optarg); break;
            case 'm': mask = atoi(optarg); break;
            case 'l': lse = atoi(optarg); break;
            case 'w': warmup = atoi(optarg); break;
            case 'i': iters = atoi(optarg); break;
            case 0: usage(argv[0]); return 0;
            default: usage(argv[0]); return 1;
        }
    }
    if (hdim != 64) {
        fprintf(stderr, "Error: this kernel is specialised for head_dim 64\n");
        return 1;
    }
    if (kv_heads == 0) kv_heads = heads;
    if (heads % kv_heads != 0) {
        fprintf(stderr, "Error: q_heads (%d) must be divisible by kv_heads (%d)\n", heads, kv_heads);
        return 1;
    }
    const bool vl = !varlen.empty();
    long long total = 0;
    if (vl) {
        batch = (int)varlen.size();
        seq = 0;
        for (int s : varlen) {
            total += s;
            seq = s > seq ? s : seq;
        }
    }
    const int D = 64;
    const size_t nq = vl ? (size_t)heads * total * D : (size_t)batch * heads * seq * D;
    const size_t nk = vl ? (size_t)kv_heads * total * D : (size_t)batch * kv_heads * seq * D;
    std::vector<uint16_t> hq(nq), hk(nk), hv(nk);
    srand(42);
    for (auto* buf : {&hq, &hk, &hv})
        for (auto& x : *buf) x = f2bf_trunc(((rand() % 1000) - 500) / 5000.0f);

    uint16_t *q, *k, *v, *o;
    float* l = nullptr;
    int32_t* ss = nullptr;
    CUDA_CHECK(cudaMalloc(&q, nq * 2));
    CUDA_CHECK(cudaMalloc(&k, nk * 2));
    CUDA_CHECK(cudaMalloc(&v, nk * 2));
    CUDA_CHECK(cudaMalloc(&o, nq * 2));
    CUDA_CHECK(cudaMemcpy(q, hq.data(), nq * 2, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(k, hk.data(), nk * 2, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(v, hv.data(), nk * 2, cudaMemcpyHostToDevice));
    if (lse) CUDA_CHECK(cudaMalloc(&l, nq / D * 4));

    FmhaFwdParams p;
    memset(&p, 0, sizeof(p));
    p.q = q; p.k = k; p.v = v; p.o = o; p.lse = l;
    p.seqlen_q = p.seqlen_k = seq;
    p.nhead_q = heads;
    p.nhead_k = kv_heads;
    p.scale = 1.4426950408889634f / sqrtf(64.0f);
    p.stride_q = p.stride_k = p.stride_v = p.stride_o = D;
    if (vl) {
        std::vector<int32_t> h(batch + 1, 0);
        for (int b = 0; b < batch; ++b) h[b + 1] = h[b] + varlen[b];
        CUDA_CHECK(cudaMalloc(&ss, (batch + 1) * 4));
        CUDA_CHECK(cudaMemcpy(ss, h.data(), (batch + 1) * 4, cudaMemcpyHostToDevice));
        p.nhead_stride_q = p.nhead_stride_o = (int)(total * D);
        p.nhead_stride_k = p.nhead_stride_v = (int)(total * D);
        p.seqstart_q = p.seqstart_k = ss;
    } else {
        p.nhead_stride_q = p.nhead_stride_o = seq * D;
        p.nhead_stride_k = p.nhead_stride_v = seq * D;
        p.batch_stride_q = p.batch_stride_o = heads * seq * D;
        p.batch_stride_k = p.batch_stride_v = kv_heads * seq * D;
    }
    auto launch = [&]() {
        return fmha_fwd_d64_bf16(&p, batch, mask, (int)total, (int)total, nullptr);
    };
    for (int i = 0; i < warmup; ++i) {
        int st = launch();
        if (st != FMHA_OK) {
            fprintf(stderr, "launch failed: %s\n", fmha_fwd_d64_error_string(st));
            return 1;
        }
    }
    CUDA_CHECK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CUDA_CHECK(cudaEventCreate(&e0));
    CUDA_CHECK(cudaEventCreate(&e1));
    std::vector<float> times(iters);
    for (int i = 0; i < iters; ++i) {
        CUDA_CHECK(cudaEventRecord(e0));
        launch();
        CUDA_CHECK(cudaEventRecord(e1));
        CUDA_CHECK(cudaEventSynchronize(e1));
        CUDA_CHECK(cudaEventElapsedTime(&times[i], e0, e1));
    }
    if (fmha_fwd_d64_status(nullptr) != FMHA_OK) {
        fprintf(stderr, "device pipeline reported an error\n");
        return 1;
    }
    float tmin = times[0], tsum = 0;
    for (float t : times) {
        tsum += t;
        tmin = t < tmin ? t : tmin;
    }
    const float tavg = tsum / iters;
    double flops;
    if (vl) {
        double s2 = 0;
        for (int s : varlen) s2 += (double)s * s;
        flops = 4.0 * heads * s2 * 64;
    } else {
        flops = 4.0 * batch * heads * (double)seq * seq * 64;
    }
    if (mask) flops *= 0.5;
    printf("Avg: %.3f ms\n", tavg);
    printf("min=%.3f ms\n", tmin);
    printf("TFLOPS: %.2f\n", flops / (tavg * 1e-3) / 1e12);
    return 0;
}
