// ref_driver.cpp -- runs the reference's own C++ port (qcau_c/src/qcau.cpp)
// on raw-binary inputs.  TEST / BASELINE INFRASTRUCTURE ONLY: it is built by
// oracle/Makefile from the reference sources where they lie (the sources are
// not copied into this repository) into oracle/_ref/qcau_ref, and is used by
// the tests to pin the oracle and by bench.py's CPU-baseline leg.
//
// Modes
//   qcau_ref attn <dir> S H C N K
//       dir/q.bin [S,H,C] bf16, dir/kv.bin [N,C] bf16, dir/idx.bin [S,K] i32,
//       dir/sink.bin [H] f32  ->  dir/out.bin [S,H,C] bf16
//       calls sparse_attention (qcau.cpp:169-284); its softmax scale is fixed
//       to 1/sqrt(C) by the reference.
//   qcau_ref qgemm <dir> S Dc N
//       dir/a.bin [S,Dc] fp8 values held as bf16 (the reference's convention,
//       main.cpp:9-24), dir/sa.bin [S,Dc/128] f32, dir/w.bin [N,Dc] bf16-held
//       fp8 values, dir/sw.bin [N/128,Dc/128] f32 -> dir/out.bin [S,N] bf16
//       calls quant_gemm (qcau.cpp:30-90).
//   qcau_ref bench_decode THREADS SEQS H C CTX DC NQ NO [STEPS [WARMUP]]
//       times one decode token per sequence: quant_gemm q-up [1,DC]x[NQ,DC],
//       sparse_attention over CTX rows with H heads of width C, quant_gemm
//       o-proj [1,H*128]x[NO,H*128]; SEQS sequences spread over THREADS
//       std::threads.  The inputs are generated before the clock starts;
//       WARMUP untimed steps, then STEPS timed ones.  Prints one JSON line
//       with the total seconds and each step's.
#include "Core.h"
#include "qcau.cpp"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

static std::vector<char> read_all(const std::string& p) {
    FILE* f = fopen(p.c_str(), "rb");
    if (!f) { fprintf(stderr, "cannot open %s\n", p.c_str()); exit(2); }
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    std::vector<char> buf(n);
    if (n && fread(buf.data(), 1, n, f) != (size_t)n) { fprintf(stderr, "short read %s\n", p.c_str()); exit(2); }
    fclose(f);
    return buf;
}

static void write_all(const std::string& p, const void* d, size_t n) {
    FILE* f = fopen(p.c_str(), "wb");
    if (!f) { fprintf(stderr, "cannot write %s\n", p.c_str()); exit(2); }
    fwrite(d, 1, n, f);
    fclose(f);
}

static int mode_attn(int argc, char** argv) {
    if (argc < 8) return 1;
    std::string dir = argv[2];
    int S = atoi(argv[3]), H = atoi(argv[4]), C = atoi(argv[5]), N = atoi(argv[6]), K = atoi(argv[7]);
    auto q = read_all(dir + "/q.bin");
    auto kv = read_all(dir + "/kv.bin");
    auto idx = read_all(dir + "/idx.bin");
    auto sink = read_all(dir + "/sink.bin");
    Tensor<__bf16> tq((__bf16*)q.data(), Shape(S, H, C), false);
    Tensor<__bf16> tkv((__bf16*)kv.data(), Shape(1, N, C), false);
    Tensor<int> tidx((int*)idx.data(), Shape(S, 1, K), false);
    Tensor<float> tsink((float*)sink.data(), Shape(1, H, 1), false);
    Tensor<__bf16> out(Shape(S, H, C));
    sparse_attention(tq, tkv, tsink, tidx, out);
    write_all(dir + "/out.bin", out.raw(), sizeof(__bf16) * (size_t)S * H * C);
    return 0;
}

static int mode_qgemm(int argc, char** argv) {
    if (argc < 6) return 1;
    std::string dir = argv[2];
    int S = atoi(argv[3]), Dc = atoi(argv[4]), N = atoi(argv[5]);
    auto a = read_all(dir + "/a.bin");
    auto sa = read_all(dir + "/sa.bin");
    auto w = read_all(dir + "/w.bin");
    auto sw = read_all(dir + "/sw.bin");
    Tensor<__bf16> ta((__bf16*)a.data(), Shape(1, S, Dc), false);
    Tensor<float> tsa((float*)sa.data(), Shape(1, S, Dc / 128), false);
    Tensor<__bf16> tw((__bf16*)w.data(), Shape(1, N, Dc), false);
    Tensor<float> tsw((float*)sw.data(), Shape(1, N / 128, Dc / 128), false);
    Tensor<__bf16> out(Shape(1, S, N));
    quant_gemm(ta, tw, tsa, tsw, true, false, out);
    write_all(dir + "/out.bin", out.raw(), sizeof(__bf16) * (size_t)S * N);
    return 0;
}

// The inputs of one decode token of one sequence, generated before any
// timing (seeded normal values, the reference's bf16-held fp8 convention for
// the GEMM operands), and the buffers its outputs go to.
struct TokenData {
    int H, C, ctx, Dc, NQ, NO;
    std::vector<__bf16> a, wq, qp, q, kv, o, ao, wo, y;
    std::vector<float> sa, swq, sink, sao, swo;
    std::vector<int> idx;

    TokenData(int H_, int C_, int ctx_, int Dc_, int NQ_, int NO_, unsigned seed)
        : H(H_), C(C_), ctx(ctx_), Dc(Dc_), NQ(NQ_), NO(NO_) {
        std::mt19937 g(seed);
        std::normal_distribution<float> nd(0.f, 1.f);
        const int no_in = H * 128;
        auto fill = [&](std::vector<__bf16>& v, size_t n, float k) {
            v.resize(n);
            for (auto& x : v) x = (__bf16)(nd(g) * k);
        };
        fill(a, (size_t)Dc, 1.f);
        sa.assign(Dc / 128, 1.0f / 64);
        fill(wq, (size_t)NQ * Dc, 8.f);
        swq.assign((size_t)(NQ / 128) * (Dc / 128), 1.0f / 512);
        qp.assign(NQ, (__bf16)0.f);
        fill(q, (size_t)H * C, 1.f);
        fill(kv, (size_t)ctx * C, 1.f);
        idx.resize(ctx);
        for (int i = 0; i < ctx; i++) idx[i] = i;
        sink.assign(H, -1e30f);
        o.assign((size_t)H * C, (__bf16)0.f);
        fill(ao, (size_t)no_in, 1.f);
        sao.assign(no_in / 128, 1.0f / 64);
        fill(wo, (size_t)NO * no_in, 8.f);
        swo.assign((size_t)(NO / 128) * (no_in / 128), 1.0f / 512);
        y.assign(NO, (__bf16)0.f);
    }

    // The reference's work for the token: quant_gemm q-up (qcau.cpp:30-90),
    // sparse_attention over all ctx rows (qcau.cpp:169-284), quant_gemm o-proj.
    void run() {
        const int no_in = H * 128;
        Tensor<__bf16> ta(a.data(), Shape(1, 1, Dc), false);
        Tensor<float> tsa(sa.data(), Shape(1, 1, Dc / 128), false);
        Tensor<__bf16> twq(wq.data(), Shape(1, NQ, Dc), false);
        Tensor<float> tswq(swq.data(), Shape(1, NQ / 128, Dc / 128), false);
        Tensor<__bf16> tqp(qp.data(), Shape(1, 1, NQ), false);
        quant_gemm(ta, twq, tsa, tswq, true, false, tqp);
        Tensor<__bf16> tq(q.data(), Shape(1, H, C), false);
        Tensor<__bf16> tkv(kv.data(), Shape(1, ctx, C), false);
        Tensor<int> tidx(idx.data(), Shape(1, 1, ctx), false);
        Tensor<float> tsink(sink.data(), Shape(1, H, 1), false);
        Tensor<__bf16> to(o.data(), Shape(1, H, C), false);
        sparse_attention(tq, tkv, tsink, tidx, to);
        Tensor<__bf16> tao(ao.data(), Shape(1, 1, no_in), false);
        Tensor<float> tsao(sao.data(), Shape(1, 1, no_in / 128), false);
        Tensor<__bf16> two(wo.data(), Shape(1, NO, no_in), false);
        Tensor<float> tswo(swo.data(), Shape(1, NO / 128, no_in / 128), false);
        Tensor<__bf16> ty(y.data(), Shape(1, 1, NO), false);
        quant_gemm(tao, two, tsao, tswo, true, false, ty);
    }
};

// Every thread builds the inputs of its sequences first; the clock runs only
// over the reference's compute.  WARMUP untimed steps, then STEPS timed ones;
// a step is one decode token of each of SEQS sequences over THREADS threads.
static int mode_bench_decode(int argc, char** argv) {
    if (argc < 10) return 1;
    int threads = atoi(argv[2]), seqs = atoi(argv[3]), H = atoi(argv[4]), C = atoi(argv[5]);
    int ctx = atoi(argv[6]), Dc = atoi(argv[7]), NQ = atoi(argv[8]), NO = atoi(argv[9]);
    int steps = argc > 10 ? atoi(argv[10]) : 1, warmup = argc > 11 ? atoi(argv[11]) : 0;
    std::vector<std::vector<TokenData>> data(threads);
    {
        std::vector<std::thread> pool;
        for (int t = 0; t < threads; t++)
            pool.emplace_back([&, t]() {
                for (int s = t; s < seqs; s += threads)
                    data[t].emplace_back(H, C, ctx, Dc, NQ, NO, 1234u + s);
            });
        for (auto& th : pool) th.join();
    }
    auto one_step = [&]() {
        std::vector<std::thread> pool;
        for (int t = 0; t < threads; t++)
            pool.emplace_back([&, t]() {
                for (auto& d : data[t]) d.run();
            });
        for (auto& th : pool) th.join();
    };
    for (int w = 0; w < warmup; w++) one_step();
    std::vector<double> per;
    for (int k = 0; k < steps; k++) {
        auto t0 = std::chrono::steady_clock::now();
        one_step();
        auto t1 = std::chrono::steady_clock::now();
        per.push_back(std::chrono::duration<double>(t1 - t0).count());
    }
    double sec = 0;
    for (double x : per) sec += x;
    printf("{\"seconds\": %.6f, \"steps\": %d, \"seqs\": %d, \"threads\": %d, \"step_seconds\": [",
           sec, steps, seqs, threads);
    for (size_t i = 0; i < per.size(); i++) printf("%s%.6f", i ? ", " : "", per[i]);
    printf("]}\n");
    return 0;
}

int main(int argc, char** argv) {
    if (argc < 2) { fprintf(stderr, "usage: qcau_ref attn|qgemm|bench_decode ...\n"); return 1; }
    std::string m = argv[1];
    int rc = 1;
    if (m == "attn") rc = mode_attn(argc, argv);
    else if (m == "qgemm") rc = mode_qgemm(argc, argv);
    else if (m == "bench_decode") rc = mode_bench_decode(argc, argv);
    if (rc) fprintf(stderr, "bad arguments for mode %s\n", m.c_str());
    return rc;
}
