// upload.cuh -- host -> device copies of a model's tensors through pinned
// staging (the loader's path, src/gguf.c:733-795 + src/forward.c:318-455: the
// reference maps a GGUF and reads tensors in place; here they cross to HBM).
#pragma once

#include <cstddef>
#include <cuda_runtime.h>
#include <vector>

namespace sllm {

// Two pinned buffers of kStageBytes. While the device copies one buffer in
// (an async copy on the uploader's stream), host threads fill the other from
// the source tensors. Small tensors are packed into one buffer and go up with
// one copy each from it. Copies larger than a buffer stream through both in
// turn. finish() waits for the last copy and reports the first error.
class Uploader {
public:
    static constexpr size_t kStageBytes = 64u << 20;
    explicit Uploader(int device);
    ~Uploader();
    // queue a copy of `bytes` from host `src` to device `dst`
    cudaError_t put(void* dst, const void* src, size_t bytes);
    cudaError_t finish();
    size_t bytes() const { return total_; }

private:
    struct Piece { void* dst; size_t off; size_t n; };
    cudaError_t flush();             // send the current buffer's pieces
    cudaError_t acquire();           // make the current buffer free to fill
    cudaStream_t stream_ = nullptr;
    unsigned char* buf_[2] = {nullptr, nullptr};
    cudaEvent_t done_[2] = {nullptr, nullptr};
    bool busy_[2] = {false, false};
    int cur_ = 0;
    size_t used_ = 0;
    std::vector<Piece> pieces_;
    cudaError_t err_ = cudaSuccess;
    size_t total_ = 0;
};

}  // namespace sllm
