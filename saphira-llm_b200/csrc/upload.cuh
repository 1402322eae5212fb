// upload.cuh -- host -> device copies of a model's tensors through pinned
// staging (the loader's path, src/gguf.c:733-795 + src/forward.c:318-455: the
// reference maps a GGUF and reads tensors in place; here they cross to HBM).
#pragma once

#include <cstddef>
#include <cuda_runtime.h>
#include <vector>

namespace sllm {

// Two pinned buffers of kStageBytes. Queued copies are packed into the
// current buffer's batch without being touched; when the batch is full, a
// team of host threads copies it into the buffer (each thread a contiguous
// share of the batch's bytes, whatever the tensor boundaries), and one async
// copy per piece sends it up while the next batch fills the other buffer.
// Copies larger than a buffer stream through both in turn. finish() sends the
// last batch, waits, and reports the first error.
class Uploader {
public:
    static constexpr size_t kStageBytes = 64u << 20;
    explicit Uploader(int device);
    ~Uploader();
    // queue a copy of `bytes` from host `src` to device `dst`. The source is
    // read when its batch is sent (by finish() at the latest) and must stay
    // valid until then, unless `transient`: then it is copied into the
    // staging buffer before put returns and may be reused at once.
    cudaError_t put(void* dst, const void* src, size_t bytes, bool transient = false);
    cudaError_t finish();
    size_t bytes() const { return total_; }

private:
    struct Piece { void* dst; const void* src; size_t off; size_t n; };   // src null: already in the buffer
    cudaError_t flush();             // fill the current buffer and send its pieces
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
