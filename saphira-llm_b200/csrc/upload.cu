// upload.cu -- pinned, double-buffered host -> device staging (upload.cuh).
#include "upload.cuh"

#include <algorithm>
#include <cstring>
#include <thread>

namespace sllm {

namespace {

// a large host copy split over a few threads (one thread moves ~10 GB/s)
void parallel_memcpy(unsigned char* dst, const unsigned char* src, size_t n) {
    constexpr size_t kMinPerThread = 4u << 20;
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t t = std::min<size_t>({(size_t)8, (size_t)hw, std::max<size_t>(1, n / kMinPerThread)});
    if (t <= 1) {
        std::memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> ths;
    const size_t per = (n + t - 1) / t;
    for (size_t i = 1; i < t; ++i) {
        const size_t a = i * per, b = std::min(n, a + per);
        if (a < b) ths.emplace_back([=] { std::memcpy(dst + a, src + a, b - a); });
    }
    std::memcpy(dst, src, std::min(n, per));
    for (auto& th : ths) th.join();
}

}  // namespace

Uploader::Uploader(int device) {
    err_ = cudaSetDevice(device);
    if (err_ == cudaSuccess) err_ = cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
    for (int i = 0; i < 2 && err_ == cudaSuccess; ++i) {
        err_ = cudaMallocHost((void**)&buf_[i], kStageBytes);
        if (err_ == cudaSuccess) err_ = cudaEventCreateWithFlags(&done_[i], cudaEventDisableTiming);
    }
}

Uploader::~Uploader() {
    if (stream_ != nullptr) cudaStreamSynchronize(stream_);
    for (int i = 0; i < 2; ++i) {
        if (buf_[i] != nullptr) cudaFreeHost(buf_[i]);
        if (done_[i] != nullptr) cudaEventDestroy(done_[i]);
    }
    if (stream_ != nullptr) cudaStreamDestroy(stream_);
}

cudaError_t Uploader::acquire() {
    if (busy_[cur_]) {
        const cudaError_t e = cudaEventSynchronize(done_[cur_]);
        if (e != cudaSuccess) return e;
        busy_[cur_] = false;
    }
    return cudaSuccess;
}

cudaError_t Uploader::flush() {
    if (pieces_.empty()) return cudaSuccess;
    for (const Piece& p : pieces_) {
        const cudaError_t e = cudaMemcpyAsync(p.dst, buf_[cur_] + p.off, p.n, cudaMemcpyHostToDevice, stream_);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = cudaEventRecord(done_[cur_], stream_);
    if (e != cudaSuccess) return e;
    busy_[cur_] = true;
    pieces_.clear();
    used_ = 0;
    cur_ ^= 1;
    return acquire();
}

cudaError_t Uploader::put(void* dst, const void* src, size_t bytes) {
    if (err_ != cudaSuccess) return err_;
    total_ += bytes;
    auto* d = static_cast<unsigned char*>(dst);
    const auto* s = static_cast<const unsigned char*>(src);
    while (bytes > 0) {
        if (used_ == kStageBytes && (err_ = flush()) != cudaSuccess) return err_;
        // 256-byte alignment of each piece inside the buffer keeps the copies fast
        const size_t n = std::min(bytes, kStageBytes - used_);
        parallel_memcpy(buf_[cur_] + used_, s, n);
        pieces_.push_back(Piece{d, used_, n});
        used_ = std::min(kStageBytes, (used_ + n + 255) & ~(size_t)255);
        d += n;
        s += n;
        bytes -= n;
    }
    return cudaSuccess;
}

cudaError_t Uploader::finish() {
    if (err_ == cudaSuccess) err_ = flush();
    if (err_ == cudaSuccess) err_ = cudaStreamSynchronize(stream_);
    return err_;
}

}  // namespace sllm
