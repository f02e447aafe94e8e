// tensor_selftest.cpp — exercises every method of the Tensor API (tensor.h,
// mirroring the reference's src/tensor.h) on the GPU and checks each result
// against a host computation.  Exit code 0 when all checks pass.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <string>
#include <utility>
#include <vector>

#include "memory_pool.h"
#include "tensor.h"

using cudasep::DType;
using cudasep::Tensor;

static int g_fail = 0;

static void expect(bool ok, const std::string& what) {
    if (!ok) {
        std::printf("FAIL %s\n", what.c_str());
        ++g_fail;
    }
}

static bool near(const std::vector<float>& a, const std::vector<float>& b, float tol = 1e-6f) {
    if (a.size() != b.size()) return false;
    for (size_t i = 0; i < a.size(); ++i)
        if (std::fabs(a[i] - b[i]) > tol * std::max(1.0f, std::fabs(b[i]))) return false;
    return true;
}

static std::vector<float> iota(int n, float s = 0.f) {
    std::vector<float> v(n);
    for (int i = 0; i < n; ++i) v[i] = s + (float)i;
    return v;
}

int main() {
    // factories and transfer
    std::vector<float> h = iota(24);
    Tensor a = Tensor::from_cpu_f32(h.data(), {2, 3, 4});
    expect(a.numel() == 24 && a.ndim() == 3 && a.size(-1) == 4 && a.is_contiguous(), "shape");
    expect(near(a.to_cpu_f32(), h), "from_cpu/to_cpu");
    expect(near(Tensor::zeros({5}).to_cpu_f32(), std::vector<float>(5, 0.f)), "zeros");
    expect(near(Tensor::ones({3}, DType::Float16).to_cpu_f32(), std::vector<float>(3, 1.f)), "ones f16");
    expect(near(Tensor::full({4}, 2.5f, DType::BFloat16).to_cpu_f32(), std::vector<float>(4, 2.5f)), "full bf16");
    expect(near(Tensor::arange(3, 8).to_cpu_f32(), iota(5, 3.f)), "arange");
    std::vector<int64_t> hi = {5, -3, 7};
    Tensor ti = Tensor::from_cpu_i64(hi.data(), {3});
    std::vector<int64_t> back(3);
    ti.copy_to_cpu(back.data(), 24);
    expect(back == hi, "i64 roundtrip");

    // views
    Tensor p = a.permute({2, 0, 1});  // [4, 2, 3]
    std::vector<float> ph(24);
    for (int k = 0; k < 4; ++k)
        for (int i = 0; i < 2; ++i)
            for (int j = 0; j < 3; ++j) ph[(k * 2 + i) * 3 + j] = h[(i * 3 + j) * 4 + k];
    expect(!p.is_contiguous() && near(p.contiguous().to_cpu_f32(), ph), "permute+contiguous");
    expect(near(p.reshape({4, -1}).to_cpu_f32(), ph), "reshape non-contiguous");
    expect(near(a.transpose(0, 2).transpose(0, 2).contiguous().to_cpu_f32(), h), "transpose twice");
    expect(a.unsqueeze(1).ndim() == 4 && a.unsqueeze(1).squeeze(1).shape() == a.shape(), "unsqueeze/squeeze");
    Tensor s = a.slice(2, 1, 3);  // [2,3,2]
    std::vector<float> sh;
    for (int i = 0; i < 6; ++i)
        for (int k = 1; k < 3; ++k) sh.push_back(h[i * 4 + k]);
    expect(near(s.contiguous().to_cpu_f32(), sh), "slice");
    expect(near(a.slice(0, -1, 2).contiguous().to_cpu_f32(), std::vector<float>(h.begin() + 12, h.end())),
           "slice negative");
    Tensor col = Tensor::from_cpu_f32(iota(3).data(), {3, 1});
    std::vector<float> eh;
    for (int i = 0; i < 3; ++i)
        for (int k = 0; k < 4; ++k) eh.push_back((float)i);
    expect(near(col.expand({3, 4}).contiguous().to_cpu_f32(), eh), "expand");
    std::vector<int64_t> idx = {3, 0, 3};
    Tensor sel = a.index_select(2, Tensor::from_cpu_i64(idx.data(), {3}));
    std::vector<float> selh;
    for (int i = 0; i < 6; ++i)
        for (int64_t k : idx) selh.push_back(h[i * 4 + k]);
    expect(near(sel.to_cpu_f32(), selh), "index_select");

    // cat / stack / split / unbind
    Tensor c = Tensor::cat({a, a.slice(2, 0, 1)}, 2);  // [2,3,5]
    std::vector<float> ch;
    for (int i = 0; i < 6; ++i) {
        for (int k = 0; k < 4; ++k) ch.push_back(h[i * 4 + k]);
        ch.push_back(h[i * 4]);
    }
    expect(c.size(2) == 5 && near(c.to_cpu_f32(), ch), "cat");
    Tensor st = Tensor::stack({a, a}, 0);
    expect(st.size(0) == 2 && near(st.slice(0, 1, 2).contiguous().to_cpu_f32(), h), "stack");
    auto parts = a.split(2, {1, 3});
    expect(parts.size() == 2 && parts[1].size(2) == 3, "split");
    auto ub = a.unbind(0);
    expect(ub.size() == 2 && near(ub[1].contiguous().to_cpu_f32(), std::vector<float>(h.begin() + 12, h.end())),
           "unbind");

    // padding
    std::vector<float> x5 = {1, 2, 3, 4, 5};
    Tensor t5 = Tensor::from_cpu_f32(x5.data(), {1, 5});
    expect(near(t5.pad({2, 1}, -1.f).to_cpu_f32(), {-1, -1, 1, 2, 3, 4, 5, -1}), "pad");
    expect(near(t5.pad_reflect({2, 3}).to_cpu_f32(), {3, 2, 1, 2, 3, 4, 5, 4, 3, 2}), "pad_reflect");

    // dtype conversion
    Tensor hb = a.to_bf16();
    expect(hb.dtype() == DType::BFloat16 && near(hb.to_f32().to_cpu_f32(), h), "to_bf16 exact ints");
    expect(near(a.to_f16().to_f32().to_cpu_f32(), h), "to_f16 exact ints");

    // arithmetic with broadcasting
    Tensor row = Tensor::from_cpu_f32(iota(4, 1.f).data(), {4});
    std::vector<float> add, mul, div;
    for (int i = 0; i < 24; ++i) {
        add.push_back(h[i] + (float)(i % 4 + 1));
        mul.push_back(h[i] * (float)(i % 4 + 1));
        div.push_back(h[i] / (float)(i % 4 + 1));
    }
    expect(near((a + row).to_cpu_f32(), add), "add broadcast");
    expect(near((a * row).to_cpu_f32(), mul), "mul broadcast");
    expect(near((a / row).to_cpu_f32(), div), "div broadcast");
    expect(near((a - a).to_cpu_f32(), std::vector<float>(24, 0.f)), "sub");
    std::vector<float> neg(24);
    for (int i = 0; i < 24; ++i) neg[i] = -h[i];
    expect(near((-a).to_cpu_f32(), neg), "neg");
    Tensor b = a.clone();
    b.add_(row);
    expect(near(b.to_cpu_f32(), add), "add_");
    b = a.clone();
    b.mul_(row);
    expect(near(b.to_cpu_f32(), mul), "mul_");
    b = a.clone();
    b.add_scalar_(1.5f).mul_scalar_(2.f).clamp_(4.f, 20.f);
    std::vector<float> sc(24);
    for (int i = 0; i < 24; ++i) sc[i] = std::min(20.f, std::max(4.f, (h[i] + 1.5f) * 2.f));
    expect(near(b.to_cpu_f32(), sc), "scalar ops");
    std::vector<float> gt(24);
    for (int i = 0; i < 24; ++i) gt[i] = h[i] > 10.f ? 1.f : 0.f;
    expect(near((a > 10.f).to_cpu_f32(), gt), "greater_than");
    b.fill_(7.f);
    expect(near(b.to_cpu_f32(), std::vector<float>(24, 7.f)), "fill_");

    // reductions
    std::vector<float> s2(6), m2(6), mx(6);
    for (int i = 0; i < 6; ++i) {
        float acc = 0, m = -1e30f;
        for (int k = 0; k < 4; ++k) {
            acc += h[i * 4 + k];
            m = std::max(m, h[i * 4 + k]);
        }
        s2[i] = acc;
        m2[i] = acc / 4;
        mx[i] = m;
    }
    expect(near(a.sum(-1).to_cpu_f32(), s2), "sum");
    expect(near(a.mean(2).to_cpu_f32(), m2), "mean");
    expect(near(a.max(2, true).to_cpu_f32(), mx) && a.max(2, true).ndim() == 3, "max keepdim");
    std::vector<float> s0(12);
    for (int j = 0; j < 12; ++j) s0[j] = h[j] + h[12 + j];
    expect(near(a.sum(0).to_cpu_f32(), s0), "sum dim0");

    // vectorised paths (contiguous operands of one dtype, 16-byte vectors,
    // tails, row / scalar broadcast, warp-per-row and column reductions),
    // checked per dtype against host arithmetic on the stored values
    for (DType dt : {DType::Float32, DType::Float16, DType::BFloat16}) {
        const std::string tn = dt == DType::Float32 ? "f32" : dt == DType::Float16 ? "f16" : "bf16";
        const float tol = dt == DType::Float32 ? 1e-5f : dt == DType::Float16 ? 2e-3f : 1.6e-2f;
        // 70: rows not a multiple of 8 elements (vector tails / scalar rows);
        // 1003 x 72: a partial group of 8 rows and odd 16-bit transposes;
        // 999 x 33: odd sizes everywhere
        for (auto rc : {std::pair<int, int>{1000, 64}, {1000, 70}, {1003, 72}, {999, 33}}) {
            const int rows = rc.first, cols = rc.second, n = rows * cols;
            std::vector<float> hx(n), hy(n), hr(cols);
            for (int i = 0; i < n; ++i) {
                hx[i] = (float)((i * 37) % 101) / 16.0f - 3.0f;  // exact in every dtype
                hy[i] = (float)((i * 53) % 89) / 32.0f + 0.5f;
            }
            for (int k = 0; k < cols; ++k) hr[k] = (float)(k % 7) / 4.0f + 1.0f;
            Tensor x = Tensor::from_cpu_f32(hx.data(), {rows, cols}).to_dtype(dt);
            Tensor y = Tensor::from_cpu_f32(hy.data(), {rows, cols}).to_dtype(dt);
            Tensor r = Tensor::from_cpu_f32(hr.data(), {cols}).to_dtype(dt);
            Tensor s1 = Tensor::full({1}, 0.75f, dt);
            const std::string tag = " " + tn + " [" + std::to_string(rows) + " x " + std::to_string(cols) + "]";
            std::vector<float> e_add(n), e_div(n), e_row(n), e_sc(n), e_cl(n);
            for (int i = 0; i < n; ++i) {
                e_add[i] = hx[i] + hy[i];
                e_div[i] = hx[i] / hy[i];
                e_row[i] = hx[i] * hr[i % cols];
                e_sc[i] = hx[i] - 0.75f;
                e_cl[i] = std::min(1.0f, std::max(-1.0f, hx[i] * 0.5f));
            }
            expect(near((x + y).to_f32().to_cpu_f32(), e_add, tol), "vec add" + tag);
            expect(near((x / y).to_f32().to_cpu_f32(), e_div, tol), "vec div" + tag);
            expect(near((x * r).to_f32().to_cpu_f32(), e_row, tol), "vec row broadcast" + tag);
            expect(near((x - s1).to_f32().to_cpu_f32(), e_sc, tol), "vec scalar broadcast" + tag);
            Tensor xc = x.clone();
            xc.mul_scalar_(0.5f).clamp_(-1.0f, 1.0f);
            expect(near(xc.to_f32().to_cpu_f32(), e_cl, tol), "vec scalar ops" + tag);
            expect(near(x.to_f32().to_cpu_f32(), hx, 0.f), "vec convert" + tag);
            std::vector<float> e_sum(rows), e_max(rows), e_col(cols, 0.f), e_cmax(cols, -1e30f);
            for (int i = 0; i < rows; ++i) {
                float acc = 0.f, m = -1e30f;
                for (int k = 0; k < cols; ++k) {
                    acc += hx[i * cols + k];
                    m = std::max(m, hx[i * cols + k]);
                    e_col[k] += hx[i * cols + k];
                    e_cmax[k] = std::max(e_cmax[k], hx[i * cols + k]);
                }
                e_sum[i] = acc;
                e_max[i] = m;
            }
            // sums are rounded once to the output dtype: compare relative to the sum's scale
            const float stol = dt == DType::Float32 ? 1e-4f : dt == DType::Float16 ? 1e-3f : 8e-3f;
            expect(near(x.sum(-1).to_f32().to_cpu_f32(), e_sum, stol), "row sum" + tag);
            expect(near(x.max(-1).to_f32().to_cpu_f32(), e_max, 0.f), "row max" + tag);
            expect(near(x.sum(0).to_f32().to_cpu_f32(), e_col, stol), "column sum" + tag);
            expect(near(x.max(0).to_f32().to_cpu_f32(), e_cmax, 0.f), "column max" + tag);
            std::vector<float> e_t((size_t)n);
            for (int i = 0; i < rows; ++i)
                for (int k = 0; k < cols; ++k) e_t[(size_t)k * rows + i] = hx[(size_t)i * cols + k];
            expect(near(x.transpose(0, 1).contiguous().to_f32().to_cpu_f32(), e_t, 0.f), "2-D transpose" + tag);
        }
    }

    // stream order of the pool: a block freed on one stream and taken on
    // another is handed over behind an event, with no host wait
    {
        cudaStream_t s1, s2;
        CUDA_CHECK(cudaStreamCreateWithFlags(&s1, cudaStreamNonBlocking));
        CUDA_CHECK(cudaStreamCreateWithFlags(&s2, cudaStreamNonBlocking));
        auto& pool = cudasep::CudaMemoryPool::instance();
        const size_t nb = 3 << 20;
        void* p = pool.allocate(nb, s1);
        CUDA_CHECK(cudaMemsetAsync(p, 0x11, nb, s1));
        pool.deallocate(p, s1);
        const auto st0 = pool.get_stats();
        void* q = pool.allocate(nb, s2);
        const auto st1 = pool.get_stats();
        expect(q == p && st1.cross_stream_reuses == st0.cross_stream_reuses + 1, "pool cross-stream reuse");
        CUDA_CHECK(cudaMemsetAsync(q, 0x22, nb, s2));
        std::vector<unsigned char> back(nb);
        CUDA_CHECK(cudaMemcpyAsync(back.data(), q, nb, cudaMemcpyDeviceToHost, s2));
        CUDA_CHECK(cudaStreamSynchronize(s2));
        bool all22 = true;
        for (unsigned char c : back) all22 = all22 && c == 0x22;
        expect(all22, "pool cross-stream reuse ordered behind the free");
        pool.deallocate(q, s2);
        void* r2 = pool.allocate(nb, s2);  // same stream: no event wait
        expect(r2 == q && pool.get_stats().cross_stream_reuses == st1.cross_stream_reuses, "pool same-stream reuse");
        pool.deallocate(r2, s2);
        CUDA_CHECK(cudaStreamSynchronize(s2));
        CUDA_CHECK(cudaStreamDestroy(s1));
        CUDA_CHECK(cudaStreamDestroy(s2));
    }

    // copy_from
    Tensor d = Tensor::empty({24});
    d.copy_from(a);
    expect(near(d.to_cpu_f32(), h), "copy_from");

    // errors surface as exceptions
    bool threw = false;
    try {
        a.reshape({5, 5});
    } catch (const std::exception&) {
        threw = true;
    }
    expect(threw, "reshape mismatch throws");
    threw = false;
    std::vector<int64_t> badi = {9};
    try {
        a.index_select(0, Tensor::from_cpu_i64(badi.data(), {1}));
    } catch (const std::exception&) {
        threw = true;
    }
    expect(threw, "index_select out of range throws");

    // allocator reuse
    auto before = cudasep::CudaMemoryPool::instance().get_stats();
    { Tensor tmp = Tensor::empty({1000}); }
    { Tensor tmp = Tensor::empty({1000}); }
    auto after = cudasep::CudaMemoryPool::instance().get_stats();
    expect(after.cache_hits > before.cache_hits, "pool reuses a freed block");
    CUDA_CHECK(cudaDeviceSynchronize());
    std::printf(g_fail ? "tensor_selftest: %d failures\n" : "tensor_selftest: OK\n", g_fail);
    return g_fail ? 1 : 0;
}
