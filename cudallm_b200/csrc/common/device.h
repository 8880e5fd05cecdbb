// Makes an engine's device current for the lifetime of the guard (engines may live on any device while
// the calling thread's current device is another).
#pragma once

#include <cuda_runtime.h>

#include "common/check.h"

namespace cudallm {

class DeviceGuard {
public:
    explicit DeviceGuard(int dev) {
        CLLM_CUDA(cudaGetDevice(&prev_));
        if (dev != prev_) CLLM_CUDA(cudaSetDevice(dev));
        set_ = dev != prev_;
    }
    ~DeviceGuard() {
        if (set_) cudaSetDevice(prev_);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int prev_ = 0;
    bool set_ = false;
};

}  // namespace cudallm
