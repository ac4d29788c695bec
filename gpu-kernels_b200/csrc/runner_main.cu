// runner_main.cu — nvfp4_runner: the reference runner's command-line contract on
// this library (matmul/sm100_nvfp4/runner.cu:36-104).
//
//   nvfp4_runner <M> <N> <K> benchmark|verify [dir]
//
// Reads the reference's interchange files from `dir` (default "."): a_mat.bin
// [M, K/2], b_mat.bin [N, K/2] (e2m1 codes), a_scales.bin / b_scales.bin (e4m3 codes,
// blocked layout, as matmul/sm100_nvfp4/main.py:36-44 writes them).  verify writes
// c_out_b200.bin (fp16 [M, N], D = A . B^T through matmul_nvfp4_b200, the
// reference-signature entry point); benchmark prints the mean milliseconds per
// GEMM and TFLOP/s over inputs rotated to exceed 3x L2.  Exit status 0 on success.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "../../include/nvfp4_b200.h"

static bool read_file(const std::string &path, std::vector<uint8_t> &buf, size_t want, size_t alt) {
    FILE *f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    std::fseek(f, 0, SEEK_END);
    const long size = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    if (size != (long)want && size != (long)alt) {
        std::fprintf(stderr, "%s: %ld bytes, expected %zu%s\n", path.c_str(), size, want,
                     alt != want ? " or the 128-row-padded size" : "");
        std::fclose(f);
        return false;
    }
    buf.assign(alt, 0);  // scale files may omit the padding rows; they stay zero
    const size_t got = std::fread(buf.data(), 1, (size_t)size, f);
    std::fclose(f);
    return got == (size_t)size;
}

int main(int argc, char **argv) {
    if (argc < 5 || (std::string(argv[4]) != "benchmark" && std::string(argv[4]) != "verify")) {
        std::fprintf(stderr, "Usage: %s <M> <N> <K> benchmark|verify [dir]\n", argv[0]);
        return 1;
    }
    const int M = std::atoi(argv[1]), N = std::atoi(argv[2]), K = std::atoi(argv[3]);
    const std::string mode = argv[4], dir = argc > 5 ? argv[5] : ".";
    if (M < 1 || N < 8 || N % 8 || K < 64 || K % 64) {
        std::fprintf(stderr, "unsupported shape (need M>=1, N%%8==0, K%%64==0)\n");
        return 1;
    }
    const size_t pm = (size_t)(M + 127) / 128 * 128, pn = (size_t)(N + 127) / 128 * 128;
    std::vector<uint8_t> a, b, sfa, sfb;
    if (!read_file(dir + "/a_mat.bin", a, (size_t)M * K / 2, (size_t)M * K / 2) ||
        !read_file(dir + "/b_mat.bin", b, (size_t)N * K / 2, (size_t)N * K / 2) ||
        !read_file(dir + "/a_scales.bin", sfa, (size_t)M * K / 16, pm * K / 16) ||
        !read_file(dir + "/b_scales.bin", sfb, (size_t)N * K / 16, pn * K / 16)) {
        std::fprintf(stderr, "cannot read the input .bin files from %s\n", dir.c_str());
        return 1;
    }
    uint8_t *da, *db, *dsfa, *dsfb;
    void *dc;
    if (cudaMalloc(&da, a.size()) || cudaMalloc(&db, b.size()) || cudaMalloc(&dsfa, sfa.size()) ||
        cudaMalloc(&dsfb, sfb.size()) || cudaMalloc(&dc, (size_t)M * N * 2)) {
        std::fprintf(stderr, "cudaMalloc failed\n");
        return 1;
    }
    cudaMemcpy(da, a.data(), a.size(), cudaMemcpyHostToDevice);
    cudaMemcpy(db, b.data(), b.size(), cudaMemcpyHostToDevice);
    cudaMemcpy(dsfa, sfa.data(), sfa.size(), cudaMemcpyHostToDevice);
    cudaMemcpy(dsfb, sfb.data(), sfb.size(), cudaMemcpyHostToDevice);

    if (mode == "verify") {
        matmul_nvfp4_b200(dc, dsfa, dsfb, da, db, M, N, K);
        if (nvfp4_last_status() != NVFP4_OK || cudaDeviceSynchronize() != cudaSuccess ||
            nvfp4_device_status(nullptr) != NVFP4_OK) {
            std::fprintf(stderr, "GEMM failed: %s\n", nvfp4_status_string(nvfp4_last_status()));
            return 1;
        }
        std::vector<uint16_t> c((size_t)M * N);
        cudaMemcpy(c.data(), dc, c.size() * 2, cudaMemcpyDeviceToHost);
        FILE *f = std::fopen((dir + "/c_out_b200.bin").c_str(), "wb");
        if (!f || std::fwrite(c.data(), 2, c.size(), f) != c.size()) {
            std::fprintf(stderr, "cannot write c_out_b200.bin\n");
            return 1;
        }
        std::fclose(f);
        std::printf("verify: wrote %s/c_out_b200.bin\n", dir.c_str());
        return 0;
    }

    // benchmark: rotate copies of the operands so that they exceed 3x L2
    int l2 = 0;
    cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, 0);
    const size_t in_bytes = a.size() + b.size() + sfa.size() + sfb.size();
    const int sets = in_bytes >= 3 * (size_t)l2 ? 1 : (int)(3 * (size_t)l2 / in_bytes) + 1;
    std::vector<uint8_t *> pa(sets, da), pb(sets, db), psa(sets, dsfa), psb(sets, dsfb);
    for (int i = 1; i < sets; i++) {
        cudaMalloc(&pa[i], a.size());
        cudaMalloc(&pb[i], b.size());
        cudaMalloc(&psa[i], sfa.size());
        cudaMalloc(&psb[i], sfb.size());
        cudaMemcpy(pa[i], da, a.size(), cudaMemcpyDeviceToDevice);
        cudaMemcpy(pb[i], db, b.size(), cudaMemcpyDeviceToDevice);
        cudaMemcpy(psa[i], dsfa, sfa.size(), cudaMemcpyDeviceToDevice);
        cudaMemcpy(psb[i], dsfb, sfb.size(), cudaMemcpyDeviceToDevice);
    }
    const int warmup = 20, reps = 100;
    for (int i = 0; i < warmup; i++) matmul_nvfp4_b200(dc, psa[i % sets], psb[i % sets], pa[i % sets], pb[i % sets], M, N, K);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0);
    for (int i = 0; i < reps; i++) matmul_nvfp4_b200(dc, psa[i % sets], psb[i % sets], pa[i % sets], pb[i % sets], M, N, K);
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    ms /= reps;
    if (nvfp4_last_status() != NVFP4_OK || nvfp4_device_status(nullptr) != NVFP4_OK) {
        std::fprintf(stderr, "GEMM failed\n");
        return 1;
    }
    std::printf("%.6f\n", ms);
    std::fprintf(stderr, "%d x %d x %d: %.4f ms, %.1f TFLOP/s (%d rotating operand sets)\n", M, N, K, ms,
                 2.0 * M * N * K / (ms * 1e-3) / 1e12, sets);
    return 0;
}
