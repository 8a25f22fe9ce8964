// bench_fmha_fwd -- timing CLI for the B200 D64 BF16 FMHA forward, with the
// reference's command line and output lines (src/bench_fmha_fwd.cpp:43-56,
// 231-233): -b -h --kv-heads -s -d --mask --lse --varlen-seqs --warmup --iters
// and "Avg: X ms" / "min=X ms" / "TFLOPS: X".  Inputs follow the reference
// generator (glibc srand(42), ((rand()%1000)-500)/5000 truncated to bf16,
// src/runner/buffers.cpp:99-127) in the reference layouts (BHSD dense,
// [H,total,D] varlen).  Varlen FLOPs count sum_b S_b^2 (the reference counts
// max_S^2 per sequence).
//
// Additions over the reference CLI (printed after its three lines, which stay
// byte-compatible):
//   --gpus N    one problem split over N GPUs of this node (strong scaling):
//               query blocks dealt out heaviest first to the least-loaded GPU
//               (LPT), every GPU holding the full inputs and running its own
//               list through fmha_fwd_d64_bf16_tiles from its own host thread;
//               no collective.  Time = max over GPUs of the per-GPU
//               CUDA-event time.  Prints "GPUS: N" and "TFLOPS/GPU: X".
//   --peak T    dense bf16 peak in TFLOP/s for the "%peak: X" line
//               [MEASURED_PEAKS.json value of this pool, 1654.3].
//   --verify N  recompute N sampled query rows per (batch, head) on the host
//               in fp64 (softmax of the bf16 inputs, P truncated to bf16 as
//               the kernel does) and print "VERIFY: max_abs=.. rel_l2=..
//               PASS|FAIL" against the bars max-abs 2e-2, rel-L2 5e-3; a
//               failure makes the exit status 2.
#include <cuda_runtime.h>
#include <getopt.h>

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
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
           "  --iters N        Benchmark iterations [20]\n"
           "  --gpus N         Split the problem over N GPUs [1]\n"
           "  --peak T         Dense bf16 peak (TFLOP/s) for %%peak [1654.3]\n"
           "  --verify N       Check N sampled rows per (batch, head) on the host [0]\n",
           prog);
}

namespace {

struct Problem {
    int batch, heads, kv_heads, seq, mask, lse;
    std::vector<int> varlen;
    long long total;
    bool vl;
};

// Query blocks (b*heads + h, m) of 128 rows with their KV-tile cost,
// dealt heaviest first to the least-loaded of n GPUs (LPT).
std::vector<std::vector<int32_t>> partition(const Problem& P, int n) {
    struct Blk { int hb, m; long long cost; };
    std::vector<Blk> blocks;
    for (int b = 0; b < P.batch; ++b) {
        const int s = P.vl ? P.varlen[b] : P.seq;
        for (int h = 0; h < P.heads; ++h)
            for (int m = 0; m * 128 < s; ++m) {
                const int kend = P.mask ? std::min(s, m * 128 + 128) : s;
                blocks.push_back({b * P.heads + h, m, (kend + 127) / 128 + 2});
            }
    }
    std::stable_sort(blocks.begin(), blocks.end(),
                     [](const Blk& x, const Blk& y) { return x.cost > y.cost; });
    std::vector<long long> load(n, 0);
    std::vector<std::vector<int32_t>> lists(n);
    for (const Blk& bk : blocks) {
        const int r = (int)(std::min_element(load.begin(), load.end()) - load.begin());
        load[r] += bk.cost;
        lists[r].push_back(bk.hb);
        lists[r].push_back(bk.m);
    }
    return lists;
}

// Host fp64 check of sampled rows: S = q.k / 8, softmax, P truncated to
// bf16 (as the kernel's P.V operand), O = P V.
struct VerifyResult { double max_abs = 0, num = 0, den = 0; };
void verify_rows(const Problem& P, const std::vector<uint16_t>& q, const std::vector<uint16_t>& k,
                 const std::vector<uint16_t>& v, const std::vector<uint16_t>& o, int nrows,
                 VerifyResult& res) {
    const int D = 64;
    auto bf = [](uint16_t x) { uint32_t u = (uint32_t)x << 16; float f; memcpy(&f, &u, 4); return (double)f; };
    const int ratio = P.heads / P.kv_heads;
    for (int b = 0; b < P.batch; ++b) {
        const int s = P.vl ? P.varlen[b] : P.seq;
        long long off = 0;
        if (P.vl) for (int i = 0; i < b; ++i) off += P.varlen[i];
        for (int h = 0; h < P.heads; ++h) {
            const int hk = h / ratio;
            for (int r = 0; r < nrows && r < s; ++r) {
                const int i = nrows == 1 ? s - 1 : (int)((long long)r * (s - 1) / (nrows - 1));
                auto qi = [&](int d) {
                    return P.vl ? q[((size_t)h * P.total + off + i) * D + d]
                                : q[(((size_t)b * P.heads + h) * s + i) * D + d];
                };
                auto kj = [&](const std::vector<uint16_t>& t, int j, int d) {
                    return P.vl ? t[((size_t)hk * P.total + off + j) * D + d]
                                : t[(((size_t)b * P.kv_heads + hk) * s + j) * D + d];
                };
                const int lim = P.mask ? i + 1 : s;
                std::vector<double> sc(lim);
                double m = -1e300;
                for (int j = 0; j < lim; ++j) {
                    double a = 0;
                    for (int d = 0; d < D; ++d) a += bf(qi(d)) * bf(kj(k, j, d));
                    sc[j] = a / 8.0;
                    m = std::max(m, sc[j]);
                }
                double l = 0;
                for (int j = 0; j < lim; ++j) l += std::exp(sc[j] - m);
                for (int d = 0; d < D; ++d) {
                    double acc = 0;
                    for (int j = 0; j < lim; ++j) {
                        const float pf = (float)(std::exp(sc[j] - m) / l);
                        uint32_t u;
                        memcpy(&u, &pf, 4);
                        u &= 0xffff0000u;
                        float pt;
                        memcpy(&pt, &u, 4);
                        acc += pt * bf(kj(v, j, d));
                    }
                    const double got = P.vl ? bf(o[((size_t)h * P.total + off + i) * D + d])
                                             : bf(o[(((size_t)b * P.heads + h) * s + i) * D + d]);
                    res.max_abs = std::max(res.max_abs, std::fabs(got - acc));
                    res.num += (got - acc) * (got - acc);
                    res.den += acc * acc;
                }
            }
        }
    }
}

struct GpuRun {
    int dev;
    std::vector<int32_t> tiles;  // empty: the whole problem through fmha_fwd_d64_bf16
    float avg_ms = 0, min_ms = 0;
    int status = 0;
    char err[256] = {0};
};

}  // namespace

#define RUN_CHECK(x)                                                                     \
    do {                                                                                 \
        cudaError_t e_ = (x);                                                            \
        if (e_ != cudaSuccess) {                                                         \
            snprintf(g.err, sizeof(g.err), "CUDA error %s at line %d", cudaGetErrorString(e_), \
                     __LINE__);                                                          \
            g.status = 1;                                                                \
            return;                                                                      \
        }                                                                                \
    } while (0)

int main(int argc, char** argv) {
    int batch = 2, heads = 16, kv_heads = 0, seq = 4096, hdim = 64, mask = 0, lse = 0;
    int warmup = 5, iters = 20, gpus = 1, verify = 0;
    double peak = 1654.3;
    std::vector<int> varlen;
    static struct option opts[] = {
        {"varlen-seqs", required_argument, 0, 6}, {"batch", required_argument, 0, 'b'},
        {"heads", required_argument, 0, 'h'},     {"kv-heads", required_argument, 0, 1},
        {"seq", required_argument, 0, 's'},       {"hdim", required_argument, 0, 'd'},
        {"mask", required_argument, 0, 'm'},      {"lse", required_argument, 0, 'l'},
        {"warmup", required_argument, 0, 'w'},    {"iters", required_argument, 0, 'i'},
        {"gpus", required_argument, 0, 7},        {"peak", required_argument, 0, 8},
        {"verify", required_argument, 0, 9},      {"help", no_argument, 0, 0},
        {0, 0, 0, 0}};
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
            case 7: gpus = atoi(optarg); break;
            case 8: peak = atof(optarg); break;
            case 9: verify = atoi(optarg); break;
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
    int ndev = 0;
    CUDA_CHECK(cudaGetDeviceCount(&ndev));
    if (gpus < 1 || gpus > ndev) {
        fprintf(stderr, "Error: --gpus %d but %d device(s) visible\n", gpus, ndev);
        return 1;
    }
    if (iters < 1) iters = 1;
    Problem P{batch, heads, kv_heads, seq, mask, lse, varlen, 0, !varlen.empty()};
    if (P.vl) {
        P.batch = (int)varlen.size();
        P.seq = 0;
        for (int s : varlen) {
            P.total += s;
            P.seq = s > P.seq ? s : P.seq;
        }
    }
    const int D = 64;
    const size_t nq = P.vl ? (size_t)heads * P.total * D : (size_t)P.batch * heads * P.seq * D;
    const size_t nk = P.vl ? (size_t)kv_heads * P.total * D : (size_t)P.batch * kv_heads * P.seq * D;
    std::vector<uint16_t> hq(nq), hk(nk), hv(nk), ho;
    srand(42);
    for (auto* buf : {&hq, &hk, &hv})
        for (auto& x : *buf) x = f2bf_trunc(((rand() % 1000) - 500) / 5000.0f);

    std::vector<GpuRun> runs(gpus);
    if (gpus > 1) {
        auto lists = partition(P, gpus);
        for (int r = 0; r < gpus; ++r) runs[r].tiles = lists[r];
    }
    for (int r = 0; r < gpus; ++r) runs[r].dev = r;
    std::mutex mu;
    std::condition_variable cv;
    int ready = 0;
    bool go = false;
    std::vector<uint16_t> o_full;  // verification copy of O (gathered from every GPU)
    if (verify > 0) o_full.assign(nq, 0);

    auto worker = [&](GpuRun& g) {
        RUN_CHECK(cudaSetDevice(g.dev));
        uint16_t *q, *k, *v, *o;
        float* l = nullptr;
        int32_t *ss = nullptr, *tl = nullptr;
        RUN_CHECK(cudaMalloc(&q, nq * 2));
        RUN_CHECK(cudaMalloc(&k, nk * 2));
        RUN_CHECK(cudaMalloc(&v, nk * 2));
        RUN_CHECK(cudaMalloc(&o, nq * 2));
        RUN_CHECK(cudaMemset(o, 0, nq * 2));
        RUN_CHECK(cudaMemcpy(q, hq.data(), nq * 2, cudaMemcpyHostToDevice));
        RUN_CHECK(cudaMemcpy(k, hk.data(), nk * 2, cudaMemcpyHostToDevice));
        RUN_CHECK(cudaMemcpy(v, hv.data(), nk * 2, cudaMemcpyHostToDevice));
        if (P.lse) RUN_CHECK(cudaMalloc(&l, nq / D * 4));
        if (!g.tiles.empty()) {
            RUN_CHECK(cudaMalloc(&tl, g.tiles.size() * 4));
            RUN_CHECK(cudaMemcpy(tl, g.tiles.data(), g.tiles.size() * 4, cudaMemcpyHostToDevice));
        }
        FmhaFwdParams p;
        memset(&p, 0, sizeof(p));
        p.q = q; p.k = k; p.v = v; p.o = o; p.lse = l;
        p.seqlen_q = p.seqlen_k = P.seq;
        p.nhead_q = P.heads;
        p.nhead_k = P.kv_heads;
        p.scale = 1.4426950408889634f / sqrtf(64.0f);
        p.stride_q = p.stride_k = p.stride_v = p.stride_o = D;
        if (P.vl) {
            std::vector<int32_t> h(P.batch + 1, 0);
            for (int b = 0; b < P.batch; ++b) h[b + 1] = h[b] + P.varlen[b];
            RUN_CHECK(cudaMalloc(&ss, (P.batch + 1) * 4));
            RUN_CHECK(cudaMemcpy(ss, h.data(), (P.batch + 1) * 4, cudaMemcpyHostToDevice));
            p.nhead_stride_q = p.nhead_stride_o = (int)(P.total * D);
            p.nhead_stride_k = p.nhead_stride_v = (int)(P.total * D);
            p.seqstart_q = p.seqstart_k = ss;
        } else {
            p.nhead_stride_q = p.nhead_stride_o = P.seq * D;
            p.nhead_stride_k = p.nhead_stride_v = P.seq * D;
            p.batch_stride_q = p.batch_stride_o = P.heads * P.seq * D;
            p.batch_stride_k = p.batch_stride_v = P.kv_heads * P.seq * D;
        }
        const int tq = (int)P.total;
        auto launch = [&]() {
            if (tl != nullptr)
                return fmha_fwd_d64_bf16_tiles(&p, P.batch, P.mask, tq, tq, tl,
                                               (int)(g.tiles.size() / 2), nullptr);
            return fmha_fwd_d64_bf16(&p, P.batch, P.mask, tq, tq, nullptr);
        };
        for (int i = 0; i < warmup; ++i) {
            const int st = launch();
            if (st != FMHA_OK) {
                snprintf(g.err, sizeof(g.err), "launch failed: %s", fmha_fwd_d64_error_string(st));
                g.status = 1;
                break;
            }
        }
        RUN_CHECK(cudaDeviceSynchronize());
        cudaEvent_t e0, e1;
        RUN_CHECK(cudaEventCreate(&e0));
        RUN_CHECK(cudaEventCreate(&e1));
        {
            // host barrier: every GPU starts its timed launches together
            std::unique_lock<std::mutex> lk(mu);
            ++ready;
            cv.notify_all();
            cv.wait(lk, [&] { return go || ready == gpus; });
            go = true;
            cv.notify_all();
        }
        std::vector<float> times(iters);
        for (int i = 0; i < iters && g.status == 0; ++i) {
            RUN_CHECK(cudaEventRecord(e0));
            launch();
            RUN_CHECK(cudaEventRecord(e1));
            RUN_CHECK(cudaEventSynchronize(e1));
            RUN_CHECK(cudaEventElapsedTime(&times[i], e0, e1));
        }
        if (fmha_fwd_d64_status(nullptr) != FMHA_OK) {
            snprintf(g.err, sizeof(g.err), "device pipeline reported an error");
            g.status = 1;
        }
        float tmin = times[0], tsum = 0;
        for (float t : times) {
            tsum += t;
            tmin = t < tmin ? t : tmin;
        }
        g.avg_ms = tsum / iters;
        g.min_ms = tmin;
        if (verify > 0 && g.status == 0) {
            std::vector<uint16_t> mine(nq);
            RUN_CHECK(cudaMemcpy(mine.data(), o, nq * 2, cudaMemcpyDeviceToHost));
            std::lock_guard<std::mutex> lk(mu);
            if (g.tiles.empty()) {
                o_full = mine;
            } else {
                // copy this GPU's blocks into the gathered O
                for (size_t t = 0; t < g.tiles.size(); t += 2) {
                    const int hb = g.tiles[t], m = g.tiles[t + 1];
                    const int b = hb / P.heads, h = hb % P.heads;
                    const int s = P.vl ? P.varlen[b] : P.seq;
                    long long off = 0;
                    if (P.vl) for (int i = 0; i < b; ++i) off += P.varlen[i];
                    for (int i = m * 128; i < std::min(s, m * 128 + 128); ++i) {
                        const size_t row = P.vl ? ((size_t)h * P.total + off + i)
                                                : (((size_t)b * P.heads + h) * s + i);
                        memcpy(&o_full[row * D], &mine[row * D], D * 2);
                    }
                }
            }
        }
        cudaFree(q); cudaFree(k); cudaFree(v); cudaFree(o);
        if (l) cudaFree(l);
        if (ss) cudaFree(ss);
        if (tl) cudaFree(tl);
    };
    std::vector<std::thread> threads;
    for (int r = 0; r < gpus; ++r) threads.emplace_back(worker, std::ref(runs[r]));
    for (auto& t : threads) t.join();
    float tavg = 0, tmin = 0;
    for (const GpuRun& g : runs) {
        if (g.status != 0) {
            fprintf(stderr, "GPU %d: %s\n", g.dev, g.err);
            return 1;
        }
        tavg = std::max(tavg, g.avg_ms);
        tmin = std::max(tmin, g.min_ms);
    }
    double flops;
    if (P.vl) {
        double s2 = 0;
        for (int s : P.varlen) s2 += (double)s * s;
        flops = 4.0 * heads * s2 * 64;
    } else {
        flops = 4.0 * P.batch * heads * (double)P.seq * P.seq * 64;
    }
    if (mask) flops *= 0.5;
    const double tflops = flops / (tavg * 1e-3) / 1e12;
    printf("Avg: %.3f ms\n", tavg);
    printf("min=%.3f ms\n", tmin);
    printf("TFLOPS: %.2f\n", tflops);
    printf("GPUS: %d\n", gpus);
    printf("TFLOPS/GPU: %.2f\n", tflops / gpus);
    printf("%%peak: %.2f\n", 100.0 * tflops / gpus / peak);
    if (verify > 0) {
        VerifyResult vr;
        verify_rows(P, hq, hk, hv, o_full, verify, vr);
        const double rel = vr.den > 0 ? std::sqrt(vr.num / vr.den) : std::sqrt(vr.num);
        const bool pass = vr.max_abs <= 2e-2 && rel <= 5e-3;
        printf("VERIFY: max_abs=%.3g rel_l2=%.3g %s\n", vr.max_abs, rel, pass ? "PASS" : "FAIL");
        if (!pass) return 2;
    }
    return 0;
}
