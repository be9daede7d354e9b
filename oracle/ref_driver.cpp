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
//   qcau_ref bench_decode THREADS SEQS H C CTX DC NQ NO
//       times one decode token per sequence: quant_gemm q-up [1,DC]x[NQ,DC],
//       sparse_attention over CTX rows with H heads of width C, quant_gemm
//       o-proj [1,H*128]x[NO,H*128]; SEQS sequences spread over THREADS
//       std::threads.  Prints one JSON line with the seconds.
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

// One decode token of one sequence through the reference's C++ kernels.
static void one_token(int H, int C, int ctx, int Dc, int NQ, int NO, unsigned seed) {
    std::mt19937 g(seed);
    std::normal_distribution<float> nd(0.f, 1.f);
    int no_in = H * 128;
    Tensor<__bf16> a(Shape(1, 1, Dc));
    Tensor<float> sa(Shape(1, 1, Dc / 128));
    Tensor<__bf16> wq(Shape(1, NQ, Dc));
    Tensor<float> swq(Shape(1, NQ / 128, Dc / 128));
    for (int i = 0; i < Dc; i++) a.raw()[i] = (__bf16)nd(g);
    for (int i = 0; i < Dc / 128; i++) sa.raw()[i] = 1.0f / 64;
    for (long i = 0; i < (long)NQ * Dc; i++) wq.raw()[i] = (__bf16)(nd(g) * 8.0f);
    for (int i = 0; i < (NQ / 128) * (Dc / 128); i++) swq.raw()[i] = 1.0f / 512;
    Tensor<__bf16> qp(Shape(1, 1, NQ));
    quant_gemm(a, wq, sa, swq, true, false, qp);

    Tensor<__bf16> q(Shape(1, H, C));
    for (int i = 0; i < H * C; i++) q.raw()[i] = (__bf16)nd(g);
    Tensor<__bf16> kv(Shape(1, ctx, C));
    for (long i = 0; i < (long)ctx * C; i++) kv.raw()[i] = (__bf16)nd(g);
    Tensor<int> idx(Shape(1, 1, ctx));
    for (int i = 0; i < ctx; i++) idx.raw()[i] = i;
    Tensor<float> sink(Shape(1, H, 1));
    for (int i = 0; i < H; i++) sink.raw()[i] = -1e30f;
    Tensor<__bf16> o(Shape(1, H, C));
    sparse_attention(q, kv, sink, idx, o);

    Tensor<__bf16> ao(Shape(1, 1, no_in));
    for (int i = 0; i < no_in; i++) ao.raw()[i] = (__bf16)nd(g);
    Tensor<float> sao(Shape(1, 1, no_in / 128));
    for (int i = 0; i < no_in / 128; i++) sao.raw()[i] = 1.0f / 64;
    Tensor<__bf16> wo(Shape(1, NO, no_in));
    for (long i = 0; i < (long)NO * no_in; i++) wo.raw()[i] = (__bf16)(nd(g) * 8.0f);
    Tensor<float> swo(Shape(1, NO / 128, no_in / 128));
    for (int i = 0; i < (NO / 128) * (no_in / 128); i++) swo.raw()[i] = 1.0f / 512;
    Tensor<__bf16> y(Shape(1, 1, NO));
    quant_gemm(ao, wo, sao, swo, true, false, y);
}

static int mode_bench_decode(int argc, char** argv) {
    if (argc < 10) return 1;
    int threads = atoi(argv[2]), seqs = atoi(argv[3]), H = atoi(argv[4]), C = atoi(argv[5]);
    int ctx = atoi(argv[6]), Dc = atoi(argv[7]), NQ = atoi(argv[8]), NO = atoi(argv[9]);
    auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; t++) {
        pool.emplace_back([=]() {
            for (int s = t; s < seqs; s += threads) one_token(H, C, ctx, Dc, NQ, NO, 1234u + s);
        });
    }
    for (auto& th : pool) th.join();
    auto t1 = std::chrono::steady_clock::now();
    double sec = std::chrono::duration<double>(t1 - t0).count();
    printf("{\"seconds\": %.6f, \"seqs\": %d, \"threads\": %d}\n", sec, seqs, threads);
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
