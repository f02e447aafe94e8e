// tensor_bench — achieved HBM bandwidth of the Tensor API's ops (the
// reference tensor library's elementwise, broadcast, conversion and reduction
// kernels, src/tensor_cuda_tile.cu:264-338, src/tensor_cuda_glue.cu:57-559)
// over the op-sweep activations [B*801*60, D], D in {192, 384, 512},
// B in {1, 4, 8}, fp32 / fp16 / bf16.
//
// Each op runs once per repetition after an L2 flush (a 256 MiB fill and a
// 256 MiB copy, so the timed launch meets a cold L2), timed alone with CUDA
// events on the legacy default stream the Tensor API uses, after two untimed
// calls that leave the caching pool warm; GB/s counts the algorithmic bytes
// (every input read once, every output written once).
// Prints one JSON line per case.
//
//   tensor_bench [reps] [peak_gbs]
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <functional>
#include <string>
#include <vector>

#include "../csrc/tensor.h"

using cudasep::DType;
using cudasep::Tensor;

namespace {

const char* name(DType d) {
    return d == DType::Float32 ? "fp32" : d == DType::Float16 ? "fp16" : "bf16";
}

struct Timer {
    cudaEvent_t a, b;
    Timer() {
        CUDA_CHECK(cudaEventCreate(&a));
        CUDA_CHECK(cudaEventCreate(&b));
    }
    ~Timer() {
        cudaEventDestroy(a);
        cudaEventDestroy(b);
    }
};

}  // namespace

int main(int argc, char** argv) {
    const int reps = argc > 1 ? std::atoi(argv[1]) : 5;
    const double peak = argc > 2 ? std::atof(argv[2]) : 0.0;
    const int T = 801, NB = 60;
    Tensor fa = Tensor::empty({64 << 20}, DType::Float32), fb = Tensor::empty({64 << 20}, DType::Float32);
    auto flush = [&] {
        fa.fill_(1.0f);
        fb.copy_from(fa);
    };
    Timer tm;
    // spin the GPU up (clocks leave their idle state) before the first timed case
    for (int i = 0; i < 2000; ++i) fa.fill_(1.0f);
    CUDA_CHECK(cudaDeviceSynchronize());
    auto run = [&](const std::string& op, DType dt, int D, int B, double bytes, const std::function<void()>& f) {
        // warm-up: an op that returns a new tensor alternates between two
        // pool blocks (the new result is allocated before the old one is
        // released), so two calls put the pool in its steady state and no
        // timed call waits on cudaMalloc
        f();
        f();
        float total = 0.f;
        for (int r = 0; r < reps; ++r) {
            flush();
            CUDA_CHECK(cudaEventRecord(tm.a, 0));
            f();
            CUDA_CHECK(cudaEventRecord(tm.b, 0));
            CUDA_CHECK(cudaEventSynchronize(tm.b));
            float ms = 0.f;
            CUDA_CHECK(cudaEventElapsedTime(&ms, tm.a, tm.b));
            total += ms;
        }
        const double ms = total / reps, gbs = bytes / (ms * 1e-3) / 1e9;
        std::printf("{\"op\": \"%s\", \"dtype\": \"%s\", \"D\": %d, \"B\": %d, \"bytes\": %.0f, \"ms\": %.5f, "
                    "\"gbs\": %.1f, \"frac\": %.3f}\n",
                    op.c_str(), name(dt), D, B, bytes, ms, gbs, peak > 0 ? gbs / peak : 0.0);
        std::fflush(stdout);
    };
    for (DType dt : {DType::Float32, DType::Float16, DType::BFloat16}) {
        const double e = (double)cudasep::dtype_size(dt);
        for (int D : {192, 384, 512})
            for (int B : {1, 4, 8}) {
                const int64_t rows = (int64_t)B * T * NB, N = rows * D;
                Tensor a = Tensor::full({rows, D}, 0.5f, dt), b = Tensor::full({rows, D}, 0.25f, dt);
                Tensor g = Tensor::full({D}, 2.0f, dt);
                Tensor c;
                run("add", dt, D, B, 3 * N * e, [&] { c = a + b; });
                c = Tensor();
                run("add_bcast_row", dt, D, B, 2 * N * e + D * e, [&] { a.add_(g); });
                run("mul_scalar", dt, D, B, 2 * N * e, [&] { a.mul_scalar_(0.5f); });
                run("fill", dt, D, B, N * e, [&] { a.fill_(0.5f); });
                const DType other = dt == DType::Float32 ? DType::Float16 : DType::Float32;
                run(std::string("to_") + name(other), dt, D, B, N * (e + (double)cudasep::dtype_size(other)),
                    [&] { c = a.to_dtype(other); });
                c = Tensor();
                run("clone", dt, D, B, 2 * N * e, [&] { c = a.clone(); });
                c = Tensor();
                run("sum_lastdim", dt, D, B, N * e + rows * e, [&] { c = a.sum(-1); });
                run("max_lastdim", dt, D, B, N * e + rows * e, [&] { c = a.max(-1); });
                run("sum_dim0", dt, D, B, N * e + D * e, [&] { c = a.sum(0); });
                c = Tensor();
                run("contiguous_transpose", dt, D, B, 2 * N * e, [&] { c = a.transpose(0, 1).contiguous(); });
                c = Tensor();
            }
    }
    CUDA_CHECK(cudaDeviceSynchronize());
    return 0;
}
