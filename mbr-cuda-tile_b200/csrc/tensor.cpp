// tensor.cpp — Tensor host logic (shapes, views, dispatch to tensor_kernels).
// Reference interface: src/tensor.h:38-148, behaviour of src/tensor.cu:14-863.
#include "tensor.h"

#include <algorithm>
#include <iostream>
#include <sstream>

#include "common.h"
#include "memory_pool.h"
#include "tensor_kernels.h"

namespace cudasep {

namespace {

int dt_code(DType d) { return (int)d; }

void check(bool c, const std::string& m) {
    if (!c) throw std::runtime_error("Tensor: " + m);
}

int norm_dim(int d, int nd, bool allow_end = false) {
    int n = nd + (allow_end ? 1 : 0);
    if (d < 0) d += n;
    check(d >= 0 && d < n, "dim out of range");
    return d;
}

std::vector<int64_t> contiguous_strides(const std::vector<int64_t>& shape) {
    std::vector<int64_t> s(shape.size());
    int64_t acc = 1;
    for (int i = (int)shape.size() - 1; i >= 0; --i) {
        s[i] = acc;
        acc *= shape[i];
    }
    return s;
}

int64_t prod(const std::vector<int64_t>& v) {
    int64_t p = 1;
    for (auto x : v) p *= x;
    return p;
}

// Broadcast shape of a and b (numpy rules) and the element strides of each
// operand over it (0 on broadcast dims).
std::vector<int64_t> broadcast(const std::vector<int64_t>& as, const std::vector<int64_t>& ast,
                               const std::vector<int64_t>& bs, const std::vector<int64_t>& bst,
                               std::vector<int64_t>& sa, std::vector<int64_t>& sb) {
    const int nd = (int)std::max(as.size(), bs.size());
    std::vector<int64_t> out(nd);
    sa.assign(nd, 0);
    sb.assign(nd, 0);
    for (int i = 0; i < nd; ++i) {
        const int ia = i - (nd - (int)as.size()), ib = i - (nd - (int)bs.size());
        const int64_t da = ia >= 0 ? as[ia] : 1, db = ib >= 0 ? bs[ib] : 1;
        check(da == db || da == 1 || db == 1, "shapes do not broadcast");
        out[i] = std::max(da, db);
        if (ia >= 0 && da != 1) sa[i] = ast[ia];
        if (ib >= 0 && db != 1) sb[i] = bst[ib];
    }
    return out;
}

}  // namespace

Tensor::Tensor() : storage_(nullptr), data_(nullptr), numel_(0), dtype_(DType::Float32) {}

std::shared_ptr<void> Tensor::alloc_gpu(size_t bytes) {
    if (bytes == 0) return nullptr;
    void* p = CudaMemoryPool::instance().allocate(bytes);
    return std::shared_ptr<void>(p, [](void* q) { CudaMemoryPool::instance().deallocate(q); });
}

void Tensor::compute_strides() { strides_ = contiguous_strides(shape_); }

Tensor Tensor::view_as(std::vector<int64_t> shape, std::vector<int64_t> strides, void* data) const {
    Tensor t;
    t.storage_ = storage_;
    t.data_ = data;
    t.shape_ = std::move(shape);
    t.strides_ = std::move(strides);
    t.numel_ = prod(t.shape_);
    t.dtype_ = dtype_;
    return t;
}

int64_t Tensor::size(int dim) const { return shape_[norm_dim(dim, ndim())]; }

bool Tensor::is_contiguous() const {
    if (numel_ <= 1) return true;
    int64_t expected = 1;
    for (int i = ndim() - 1; i >= 0; --i) {
        if (shape_[i] != 1 && strides_[i] != expected) return false;
        expected *= shape_[i];
    }
    return true;
}

// ---- factories ----
Tensor Tensor::empty(std::vector<int64_t> shape, DType dtype) {
    Tensor t;
    for (auto s : shape) check(s >= 0, "negative size");
    t.shape_ = std::move(shape);
    t.dtype_ = dtype;
    t.numel_ = prod(t.shape_);
    t.compute_strides();
    t.storage_ = alloc_gpu((size_t)t.numel_ * dtype_size(dtype));
    t.data_ = t.storage_.get();
    return t;
}

Tensor Tensor::full(std::vector<int64_t> shape, float value, DType dtype) {
    Tensor t = empty(std::move(shape), dtype);
    t.fill_(value);
    return t;
}
Tensor Tensor::zeros(std::vector<int64_t> shape, DType dtype) { return full(std::move(shape), 0.0f, dtype); }
Tensor Tensor::ones(std::vector<int64_t> shape, DType dtype) { return full(std::move(shape), 1.0f, dtype); }

Tensor Tensor::from_cpu_f32(const float* data, std::vector<int64_t> shape) {
    Tensor t = empty(std::move(shape), DType::Float32);
    t.copy_from_cpu(data, (size_t)t.numel_ * 4);
    return t;
}
Tensor Tensor::from_cpu_f16(const void* data, std::vector<int64_t> shape) {
    Tensor t = empty(std::move(shape), DType::Float16);
    t.copy_from_cpu(data, (size_t)t.numel_ * 2);
    return t;
}
Tensor Tensor::from_cpu_i64(const int64_t* data, std::vector<int64_t> shape) {
    Tensor t = empty(std::move(shape), DType::Int64);
    t.copy_from_cpu(data, (size_t)t.numel_ * 8);
    return t;
}
Tensor Tensor::arange(int64_t start, int64_t end, DType dtype) {
    Tensor t = empty({std::max<int64_t>(0, end - start)}, dtype);
    tk::arange(t.data_, dt_code(dtype), start, t.numel_, 0);
    return t;
}

// ---- host transfer ----
void Tensor::copy_from_cpu(const void* src, size_t bytes) {
    check(is_contiguous() && bytes <= (size_t)numel_ * dtype_size(dtype_), "copy_from_cpu size/layout");
    if (bytes) CUDA_CHECK(cudaMemcpy(data_, src, bytes, cudaMemcpyHostToDevice));
}
void Tensor::copy_to_cpu(void* dst, size_t bytes) const {
    Tensor c = contiguous();
    check(bytes <= (size_t)numel_ * dtype_size(dtype_), "copy_to_cpu size");
    if (bytes) CUDA_CHECK(cudaMemcpy(dst, c.data_, bytes, cudaMemcpyDeviceToHost));
}
std::vector<float> Tensor::to_cpu_f32() const {
    Tensor f = to_dtype(DType::Float32);
    std::vector<float> v((size_t)numel_);
    f.copy_to_cpu(v.data(), v.size() * 4);
    return v;
}

// ---- views ----
Tensor Tensor::reshape(std::vector<int64_t> ns) const {
    int infer = -1;
    int64_t known = 1;
    for (size_t i = 0; i < ns.size(); ++i) {
        if (ns[i] == -1) {
            check(infer < 0, "reshape: more than one -1");
            infer = (int)i;
        } else {
            known *= ns[i];
        }
    }
    if (infer >= 0) ns[infer] = known ? numel_ / known : 0;
    check(prod(ns) == numel_, "reshape: element count mismatch " + shape_str());
    const Tensor c = contiguous();
    return c.view_as(ns, contiguous_strides(ns), c.data_);
}

Tensor Tensor::permute(std::vector<int> dims) const {
    check((int)dims.size() == ndim(), "permute: rank mismatch");
    std::vector<int64_t> sh(dims.size()), st(dims.size());
    std::vector<bool> seen(dims.size(), false);
    for (size_t i = 0; i < dims.size(); ++i) {
        int d = norm_dim(dims[i], ndim());
        check(!seen[d], "permute: repeated dim");
        seen[d] = true;
        sh[i] = shape_[d];
        st[i] = strides_[d];
    }
    return view_as(sh, st, data_);
}

Tensor Tensor::transpose(int d0, int d1) const {
    std::vector<int> p(ndim());
    for (int i = 0; i < ndim(); ++i) p[i] = i;
    std::swap(p[norm_dim(d0, ndim())], p[norm_dim(d1, ndim())]);
    return permute(p);
}

Tensor Tensor::contiguous() const {
    if (is_contiguous()) return *this;
    Tensor out = empty(shape_, dtype_);
    tk::copy(data_, dt_code(dtype_), strides_.data(), out.data_, dt_code(dtype_), out.strides_.data(), ndim(),
             shape_.data(), numel_, 0);
    return out;
}

Tensor Tensor::unsqueeze(int dim) const {
    dim = norm_dim(dim, ndim(), true);
    std::vector<int64_t> sh = shape_, st = strides_;
    int64_t s = dim < ndim() ? strides_[dim] * shape_[dim] : 1;
    sh.insert(sh.begin() + dim, 1);
    st.insert(st.begin() + dim, s);
    return view_as(sh, st, data_);
}

Tensor Tensor::squeeze(int dim) const {
    dim = norm_dim(dim, ndim());
    if (shape_[dim] != 1) return *this;
    std::vector<int64_t> sh = shape_, st = strides_;
    sh.erase(sh.begin() + dim);
    st.erase(st.begin() + dim);
    return view_as(sh, st, data_);
}

Tensor Tensor::expand(std::vector<int64_t> ns) const {
    check(ns.size() >= shape_.size(), "expand: rank");
    const int off = (int)(ns.size() - shape_.size());
    std::vector<int64_t> st(ns.size(), 0);
    for (int i = 0; i < (int)ns.size(); ++i) {
        const int j = i - off;
        if (j < 0) continue;
        if (ns[i] == -1) ns[i] = shape_[j];
        check(shape_[j] == ns[i] || shape_[j] == 1, "expand: incompatible dim");
        st[i] = shape_[j] == ns[i] ? strides_[j] : 0;
    }
    return view_as(ns, st, data_);
}

Tensor Tensor::slice(int dim, int64_t start, int64_t end) const {
    dim = norm_dim(dim, ndim());
    const int64_t n = shape_[dim];
    if (start < 0) start += n;
    if (end < 0) end += n;
    start = std::min(std::max<int64_t>(start, 0), n);
    end = std::min(std::max<int64_t>(end, start), n);
    std::vector<int64_t> sh = shape_;
    sh[dim] = end - start;
    return view_as(sh, strides_, (char*)data_ + start * strides_[dim] * (int64_t)dtype_size(dtype_));
}

Tensor Tensor::index_select(int dim, const Tensor& indices) const {
    dim = norm_dim(dim, ndim());
    check(indices.dtype() == DType::Int64 && indices.ndim() == 1, "index_select: indices must be 1-D int64");
    const Tensor c = contiguous();
    const Tensor idx = indices.contiguous();
    std::vector<int64_t> sh = shape_;
    sh[dim] = idx.numel();
    Tensor out = empty(sh, dtype_);
    int64_t outer = 1, inner = 1;
    for (int i = 0; i < dim; ++i) outer *= shape_[i];
    for (int i = dim + 1; i < ndim(); ++i) inner *= shape_[i];
    int* d_bad = nullptr;
    CUDA_CHECK(cudaMallocAsync((void**)&d_bad, sizeof(int), 0));
    CUDA_CHECK(cudaMemsetAsync(d_bad, 0, sizeof(int), 0));
    tk::index_select(c.data_, dt_code(dtype_), outer, shape_[dim], inner, (const int64_t*)idx.data_ptr(),
                     idx.numel(), out.data_, d_bad, 0);
    int bad = 0;
    CUDA_CHECK(cudaMemcpy(&bad, d_bad, sizeof(int), cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaFreeAsync(d_bad, 0));
    check(!bad, "index_select: index out of range");
    return out;
}

Tensor Tensor::cat(const std::vector<Tensor>& ts, int dim) {
    check(!ts.empty(), "cat: no tensors");
    const Tensor& f = ts[0];
    dim = norm_dim(dim, f.ndim());
    std::vector<int64_t> sh = f.shape_;
    int64_t total = 0;
    for (const Tensor& t : ts) {
        check(t.ndim() == f.ndim() && t.dtype() == f.dtype(), "cat: rank/dtype mismatch");
        for (int i = 0; i < f.ndim(); ++i)
            if (i != dim) check(t.shape_[i] == sh[i], "cat: shape mismatch");
        total += t.shape_[dim];
    }
    sh[dim] = total;
    Tensor out = empty(sh, f.dtype());
    int64_t off = 0;
    for (const Tensor& t : ts) {
        Tensor dst = out.slice(dim, off, off + t.shape_[dim]);
        tk::copy(t.data_, dt_code(t.dtype_), t.strides_.data(), dst.data_, dt_code(dst.dtype_), dst.strides_.data(),
                 t.ndim(), t.shape_.data(), t.numel_, 0);
        off += t.shape_[dim];
    }
    return out;
}

Tensor Tensor::stack(const std::vector<Tensor>& ts, int dim) {
    check(!ts.empty(), "stack: no tensors");
    std::vector<Tensor> u;
    u.reserve(ts.size());
    for (const Tensor& t : ts) u.push_back(t.unsqueeze(dim));
    return cat(u, dim);
}

std::vector<Tensor> Tensor::split(int dim, const std::vector<int64_t>& sizes) const {
    dim = norm_dim(dim, ndim());
    int64_t tot = 0;
    for (auto s : sizes) tot += s;
    check(tot == shape_[dim], "split: sizes do not sum to the dim");
    std::vector<Tensor> out;
    int64_t off = 0;
    for (auto s : sizes) {
        out.push_back(slice(dim, off, off + s));
        off += s;
    }
    return out;
}

std::vector<Tensor> Tensor::unbind(int dim) const {
    dim = norm_dim(dim, ndim());
    std::vector<Tensor> out;
    for (int64_t i = 0; i < shape_[dim]; ++i) out.push_back(slice(dim, i, i + 1).squeeze(dim));
    return out;
}

Tensor Tensor::pad(const std::vector<int64_t>& p, float value) const {
    check(p.size() == 2 && p[0] >= 0 && p[1] >= 0 && ndim() >= 1, "pad: {left, right} on the last dim");
    std::vector<int64_t> sh = shape_;
    sh.back() += p[0] + p[1];
    Tensor out = full(sh, value, dtype_);
    Tensor dst = out.slice(-1, p[0], p[0] + shape_.back());
    tk::copy(data_, dt_code(dtype_), strides_.data(), dst.data_, dt_code(dtype_), dst.strides_.data(), ndim(),
             shape_.data(), numel_, 0);
    return out;
}

Tensor Tensor::pad_reflect(const std::vector<int64_t>& p) const {
    check(p.size() == 2 && p[0] >= 0 && p[1] >= 0 && ndim() >= 1, "pad_reflect: {left, right} on the last dim");
    const int64_t L = shape_.back();
    check(p[0] < L && p[1] < L, "pad_reflect: padding must be smaller than the dim");
    const Tensor c = contiguous();
    std::vector<int64_t> sh = shape_;
    sh.back() += p[0] + p[1];
    Tensor out = empty(sh, dtype_);
    tk::pad_reflect(c.data_, dt_code(dtype_), numel_ / std::max<int64_t>(L, 1), L, p[0], p[1], out.data_, 0);
    return out;
}

Tensor Tensor::to_dtype(DType nd) const {
    if (nd == dtype_) return *this;
    Tensor out = empty(shape_, nd);
    tk::copy(data_, dt_code(dtype_), strides_.data(), out.data_, dt_code(nd), out.strides_.data(), ndim(),
             shape_.data(), numel_, 0);
    return out;
}

// ---- arithmetic ----
Tensor Tensor::binary_op(const Tensor& o, int op) const {
    std::vector<int64_t> sa, sb;
    std::vector<int64_t> sh = broadcast(shape_, strides_, o.shape_, o.strides_, sa, sb);
    DType od = (dtype_ == DType::Float32 || o.dtype_ == DType::Float32) ? DType::Float32 : dtype_;
    Tensor out = empty(sh, od);
    tk::binary(op, data_, dt_code(dtype_), sa.data(), o.data_, dt_code(o.dtype_), sb.data(), out.data_, dt_code(od),
               out.strides_.data(), (int)sh.size(), sh.data(), out.numel_, 0);
    return out;
}

Tensor& Tensor::binary_inplace(const Tensor& o, int op) {
    std::vector<int64_t> sa, sb;
    std::vector<int64_t> sh = broadcast(shape_, strides_, o.shape_, o.strides_, sa, sb);
    check(sh == shape_, "in-place op: the other tensor must broadcast to this shape");
    tk::binary(op, data_, dt_code(dtype_), sa.data(), o.data_, dt_code(o.dtype_), sb.data(), data_, dt_code(dtype_),
               strides_.data(), ndim(), shape_.data(), numel_, 0);
    return *this;
}

Tensor Tensor::operator+(const Tensor& o) const { return binary_op(o, tk::BIN_ADD); }
Tensor Tensor::operator-(const Tensor& o) const { return binary_op(o, tk::BIN_SUB); }
Tensor Tensor::operator*(const Tensor& o) const { return binary_op(o, tk::BIN_MUL); }
Tensor Tensor::operator/(const Tensor& o) const { return binary_op(o, tk::BIN_DIV); }
Tensor Tensor::operator-() const {
    Tensor out = empty(shape_, dtype_);
    tk::unary(tk::UN_NEG, data_, dt_code(dtype_), strides_.data(), out.data_, dt_code(dtype_), out.strides_.data(),
              ndim(), shape_.data(), numel_, 0.f, 0.f, 0);
    return out;
}

Tensor& Tensor::add_(const Tensor& o) { return binary_inplace(o, tk::BIN_ADD); }
Tensor& Tensor::mul_(const Tensor& o) { return binary_inplace(o, tk::BIN_MUL); }

Tensor& Tensor::add_scalar_(float v) {
    tk::unary(tk::UN_ADD_SCALAR, data_, dt_code(dtype_), strides_.data(), data_, dt_code(dtype_), strides_.data(),
              ndim(), shape_.data(), numel_, v, 0.f, 0);
    return *this;
}
Tensor& Tensor::mul_scalar_(float v) {
    tk::unary(tk::UN_MUL_SCALAR, data_, dt_code(dtype_), strides_.data(), data_, dt_code(dtype_), strides_.data(),
              ndim(), shape_.data(), numel_, v, 0.f, 0);
    return *this;
}
Tensor& Tensor::clamp_(float lo, float hi) {
    tk::unary(tk::UN_CLAMP, data_, dt_code(dtype_), strides_.data(), data_, dt_code(dtype_), strides_.data(), ndim(),
              shape_.data(), numel_, lo, hi, 0);
    return *this;
}
Tensor& Tensor::fill_(float v) {
    tk::fill(data_, dt_code(dtype_), strides_.data(), ndim(), shape_.data(), numel_, v, 0);
    return *this;
}

Tensor Tensor::operator>(float v) const {
    Tensor out = empty(shape_, DType::Float32);
    tk::unary(tk::UN_GT, data_, dt_code(dtype_), strides_.data(), out.data_, dt_code(DType::Float32),
              out.strides_.data(), ndim(), shape_.data(), numel_, v, 0.f, 0);
    return out;
}

// ---- reductions ----
Tensor Tensor::reduce_op(int dim, bool keepdim, int op) const {
    dim = norm_dim(dim, ndim());
    std::vector<int64_t> osh, ost;
    for (int i = 0; i < ndim(); ++i)
        if (i != dim) {
            osh.push_back(shape_[i]);
            ost.push_back(strides_[i]);
        }
    DType od = dtype_ == DType::Int64 ? DType::Float32 : dtype_;
    Tensor out = empty(osh, od);
    tk::reduce(op, data_, dt_code(dtype_), ost.data(), (int)osh.size(), osh.data(), out.numel_, shape_[dim],
               strides_[dim], out.data_, dt_code(od), 0);
    return keepdim ? out.unsqueeze(dim) : out;
}
Tensor Tensor::sum(int dim, bool keepdim) const { return reduce_op(dim, keepdim, tk::RED_SUM); }
Tensor Tensor::mean(int dim, bool keepdim) const { return reduce_op(dim, keepdim, tk::RED_MEAN); }
Tensor Tensor::max(int dim, bool keepdim) const { return reduce_op(dim, keepdim, tk::RED_MAX); }

// ---- copies ----
Tensor Tensor::clone() const {
    Tensor out = empty(shape_, dtype_);
    tk::copy(data_, dt_code(dtype_), strides_.data(), out.data_, dt_code(dtype_), out.strides_.data(), ndim(),
             shape_.data(), numel_, 0);
    return out;
}

void Tensor::copy_from(const Tensor& src) {
    check(src.numel_ == numel_, "copy_from: element count mismatch");
    const Tensor s = src.shape_ == shape_ ? src : src.reshape(shape_);
    tk::copy(s.data_, dt_code(s.dtype_), s.strides_.data(), data_, dt_code(dtype_), strides_.data(), ndim(),
             shape_.data(), numel_, 0);
}

// ---- debug ----
std::string Tensor::shape_str() const {
    std::ostringstream s;
    s << "[";
    for (size_t i = 0; i < shape_.size(); ++i) s << (i ? ", " : "") << shape_[i];
    s << "]";
    return s.str();
}

void Tensor::print(const std::string& name, int max_elements) const {
    std::vector<float> v = to_cpu_f32();
    std::cout << (name.empty() ? "Tensor" : name) << " " << shape_str() << " dtype=" << (int)dtype_ << " [";
    for (int i = 0; i < std::min<int64_t>(max_elements, (int64_t)v.size()); ++i) std::cout << (i ? ", " : "") << v[i];
    if ((int64_t)v.size() > max_elements) std::cout << ", ...";
    std::cout << "]" << std::endl;
}

}  // namespace cudasep
