// jhq_common.h — status codes, error type, CUDA checks and RAII buffers used
// by every translation unit of the JHQ B200 engine.
//
// The reference reports errors by exit(1) (common/cuda_utils.cuh:7-25) or by
// throwing std::invalid_argument / std::runtime_error from JHQGpuIndex
// (jhq_v14_streaming_add/jhq_gpu_index.cu:110-121, :418-420, :537). Here the
// C++ layer throws jhq::Error carrying one of the JHQ_* status codes of
// include/jhq.h, and the C-ABI turns it into a return code; nothing exits.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <mutex>
#include <utility>

#include "../../include/jhq.h"

namespace jhq {

class Error : public std::runtime_error {
public:
    Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
    int code() const { return code_; }
private:
    int code_;
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error(code, msg); }

inline void cuda_check(cudaError_t e, const char* what, const char* file, int line) {
    if (e == cudaSuccess) return;
    char buf[512];
    std::snprintf(buf, sizeof buf, "%s failed at %s:%d: %s", what, file, line, cudaGetErrorString(e));
    int code = (e == cudaErrorMemoryAllocation) ? JHQ_ENOMEM : JHQ_EDEVICE;
    throw Error(code, buf);
}
#define JHQ_CUDA(call) ::jhq::cuda_check((call), #call, __FILE__, __LINE__)
#define JHQ_LAUNCH_CHECK() ::jhq::cuda_check(cudaGetLastError(), "kernel launch", __FILE__, __LINE__)

// Scoped device selection: every public entry point runs on the index's device.
class DeviceGuard {
public:
    explicit DeviceGuard(int dev) {
        JHQ_CUDA(cudaGetDevice(&prev_));
        if (prev_ != dev) JHQ_CUDA(cudaSetDevice(dev));
        dev_ = dev;
    }
    ~DeviceGuard() { if (prev_ != dev_) cudaSetDevice(prev_); }
private:
    int prev_ = 0, dev_ = 0;
};

// Owning device allocation (cudaMalloc / cudaFree), movable, never copied.
template <class T>
class DevBuf {
public:
    DevBuf() = default;
    explicit DevBuf(size_t n) { resize(n); }
    ~DevBuf() { release(); }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr; o.n_ = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) { release(); p_ = o.p_; n_ = o.n_; o.p_ = nullptr; o.n_ = 0; }
        return *this;
    }
    void resize(size_t n) {          // contents are NOT preserved
        if (n == n_) return;
        release();
        if (n) JHQ_CUDA(cudaMalloc(reinterpret_cast<void**>(&p_), n * sizeof(T)));
        n_ = n;
    }
    void ensure(size_t n) { if (n > n_) resize(n); }   // grow-only, contents not preserved
    void release() { if (p_) cudaFree(p_); p_ = nullptr; n_ = 0; }
    T* get() const { return p_; }
    size_t size() const { return n_; }
    size_t bytes() const { return n_ * sizeof(T); }
private:
    T* p_ = nullptr;
    size_t n_ = 0;
};

// Owning pinned host allocation (cudaMallocHost / cudaFreeHost).
template <class T>
class PinnedBuf {
public:
    PinnedBuf() = default;
    ~PinnedBuf() { release(); }
    PinnedBuf(const PinnedBuf&) = delete;
    PinnedBuf& operator=(const PinnedBuf&) = delete;
    void ensure(size_t n) {
        if (n <= n_) return;
        release();
        JHQ_CUDA(cudaMallocHost(reinterpret_cast<void**>(&p_), n * sizeof(T)));
        n_ = n;
    }
    void release() { if (p_) cudaFreeHost(p_); p_ = nullptr; n_ = 0; }
    T* get() const { return p_; }
    size_t size() const { return n_; }
private:
    T* p_ = nullptr;
    size_t n_ = 0;
};

// Pinned, device-mapped host allocation (cudaHostAllocMapped: with unified
// addressing the same pointer is valid in kernels, which read it over the host
// link). Grows geometrically and keeps its first `keep` elements.
template <class T>
class MappedBuf {
public:
    MappedBuf() = default;
    ~MappedBuf() { release(); }
    MappedBuf(const MappedBuf&) = delete;
    MappedBuf& operator=(const MappedBuf&) = delete;
    void grow(size_t n, size_t keep) {
        if (n <= n_) return;
        size_t nc = n_ + n_ / 2 > n ? n_ + n_ / 2 : n;
        T* p = nullptr;
        JHQ_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&p), nc * sizeof(T),
                               cudaHostAllocMapped | cudaHostAllocPortable));
        if (p_ && keep) std::memcpy(p, p_, keep * sizeof(T));
        release();
        p_ = p;
        n_ = nc;
    }
    void release() { if (p_) cudaFreeHost(p_); p_ = nullptr; n_ = 0; }
    T* get() const { return p_; }
    size_t size() const { return n_; }
private:
    T* p_ = nullptr;
    size_t n_ = 0;
};

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Stream-ordered copies of n elements.
template <class T>
void h2d(T* dst, const T* src, size_t n, cudaStream_t s) {
    if (n) JHQ_CUDA(cudaMemcpyAsync(dst, src, n * sizeof(T), cudaMemcpyHostToDevice, s));
}
template <class T>
void d2h(T* dst, const T* src, size_t n, cudaStream_t s) {
    if (n) JHQ_CUDA(cudaMemcpyAsync(dst, src, n * sizeof(T), cudaMemcpyDeviceToHost, s));
}
inline int next_pow2(int x) { int p = 1; while (p < x) p <<= 1; return p; }

// Runs f once per CUDA device of the process, with that device current
// (function attributes such as the opt-in shared memory size are per device).
template <class F>
void once_per_device(std::atomic<uint64_t>& done, F&& f) {
    int dev = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (done.load() & bit) return;
    f();
    done.fetch_or(bit);
}

}  // namespace jhq
