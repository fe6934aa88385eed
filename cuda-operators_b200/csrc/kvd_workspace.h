// kvd_workspace.h -- stream-ordered owner of one scratch allocation.
//
// Same contract as mur::OrderedWorkspace (common/ordered_workspace.cuh:10-58 of
// the reference): the buffer is allocated with cudaMallocAsync on a stream,
// every outstanding use belongs to last_stream(), handoff(next) orders `next`
// after the current owner through an event, and close()/the destructor release
// it with cudaFreeAsync on the last stream, so freeing never synchronises the
// device. Differences: errors are reported through status() instead of
// exceptions (the owner is used behind a C ABI), and an empty request is a
// valid no-op owner instead of an error.
#pragma once

#include <cstddef>
#include <utility>
#include <cuda_runtime.h>

namespace kvd {

class OrderedWorkspace {
public:
    struct Audit {
        int allocations = 0, free_submissions = 0, cleanup_errors = 0;
    };

    OrderedWorkspace(size_t bytes, cudaStream_t stream, Audit* audit = nullptr)
        : last_(stream), audit_(audit) {
        if (bytes == 0) return;
        status_ = cudaMallocAsync(&pointer_, bytes, stream);
        if (status_ != cudaSuccess) {
            pointer_ = nullptr;
            return;
        }
        bytes_ = bytes;
        if (audit_) ++audit_->allocations;
    }
    OrderedWorkspace(const OrderedWorkspace&) = delete;
    OrderedWorkspace& operator=(const OrderedWorkspace&) = delete;
    OrderedWorkspace(OrderedWorkspace&& o) noexcept
        : pointer_(std::exchange(o.pointer_, nullptr)), bytes_(std::exchange(o.bytes_, 0)),
          last_(o.last_), audit_(o.audit_), status_(o.status_) {}
    OrderedWorkspace& operator=(OrderedWorkspace&&) = delete;

    void* data() const noexcept { return pointer_; }
    size_t bytes() const noexcept { return bytes_; }
    cudaStream_t last_stream() const noexcept { return last_; }
    cudaError_t status() const noexcept { return status_; }

    // Orders `next` after all work queued on the current owner stream.
    cudaError_t handoff(cudaStream_t next) {
        if (next == last_) return cudaSuccess;
        cudaEvent_t ev{};
        cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e != cudaSuccess) return e;
        e = cudaEventRecord(ev, last_);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(next, ev, 0);
        const cudaError_t d = cudaEventDestroy(ev);
        if (e != cudaSuccess) return e;
        last_ = next;  // the wait is queued: ownership moves even if destroy reports an error
        return d;
    }

    cudaError_t close() {
        if (!pointer_) return cudaSuccess;
        const cudaError_t e = cudaFreeAsync(pointer_, last_);
        pointer_ = nullptr;
        bytes_ = 0;
        if (audit_) {
            if (e == cudaSuccess) ++audit_->free_submissions;
            else ++audit_->cleanup_errors;
        }
        return e;
    }

    ~OrderedWorkspace() noexcept { close(); }

private:
    void* pointer_ = nullptr;
    size_t bytes_ = 0;
    cudaStream_t last_{};
    Audit* audit_ = nullptr;
    cudaError_t status_ = cudaSuccess;
};

}  // namespace kvd
