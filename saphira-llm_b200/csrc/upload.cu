// upload.cu -- pinned, double-buffered host -> device staging (upload.cuh).
#include "upload.cuh"

#include <algorithm>
#include <cstring>
#include <thread>

namespace sllm {

namespace {

// Copy the pieces' source bytes to buf + piece.off, over a few threads: the
// batch's bytes are cut into equal contiguous shares, each thread copying the
// parts of the pieces that fall in its share (one thread moves ~10 GB/s).
template <class P>
void fill_batch(unsigned char* buf, const std::vector<P>& pieces) {
    size_t total = 0;
    for (const P& p : pieces) total += p.src != nullptr ? p.n : 0;
    if (total == 0) return;
    constexpr size_t kMinPerThread = 2u << 20;
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t t = std::min<size_t>({(size_t)16, (size_t)hw, std::max<size_t>(1, total / kMinPerThread)});
    const size_t share = (total + t - 1) / t;
    auto work = [&](size_t lo, size_t hi) {        // bytes [lo, hi) of the batch, in piece order
        size_t at = 0;
        for (const P& p : pieces) {
            if (p.src == nullptr) continue;      // copied at put()
            const size_t a = std::max(lo, at), b = std::min(hi, at + p.n);
            if (a < b)
                std::memcpy(buf + p.off + (a - at), static_cast<const unsigned char*>(p.src) + (a - at), b - a);
            at += p.n;
            if (at >= hi) break;
        }
    };
    std::vector<std::thread> ths;
    for (size_t i = 1; i < t; ++i) {
        const size_t lo = i * share, hi = std::min(total, lo + share);
        if (lo < hi) ths.emplace_back(work, lo, hi);
    }
    work(0, std::min(total, share));
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
    fill_batch(buf_[cur_], pieces_);
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

cudaError_t Uploader::put(void* dst, const void* src, size_t bytes, bool transient) {
    if (err_ != cudaSuccess) return err_;
    total_ += bytes;
    auto* d = static_cast<unsigned char*>(dst);
    const auto* s = static_cast<const unsigned char*>(src);
    while (bytes > 0) {
        if (used_ == kStageBytes && (err_ = flush()) != cudaSuccess) return err_;
        // 256-byte alignment of each piece inside the buffer keeps the copies fast
        const size_t n = std::min(bytes, kStageBytes - used_);
        if (transient) std::memcpy(buf_[cur_] + used_, s, n);
        pieces_.push_back(Piece{d, transient ? nullptr : s, used_, n});
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
