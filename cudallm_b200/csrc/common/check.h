// Typed host-side errors and check macros. The C ABI maps each type to one return code, the same
// mapping as wasiqnauman/cudallm src/capi/cudallm_capi.cpp:24-30 (ArgError -> INVALID_ARG,
// FormatError -> FORMAT, IoError -> IO, a message containing "CUDA" -> CUDA, StateError -> STATE,
// anything else -> INTERNAL).
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace cudallm {

class ArgError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};
class FormatError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};
class IoError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};
class StateError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

[[noreturn]] inline void throw_cuda(cudaError_t err, const char* expr, const char* file, int line) {
    throw std::runtime_error(std::string("CUDA error at ") + file + ":" + std::to_string(line) + ": " + expr + ": " +
                             cudaGetErrorString(err));
}

}  // namespace cudallm

#define CLLM_CUDA(expr)                                                                  \
    do {                                                                                 \
        cudaError_t cllm_err_ = (expr);                                                  \
        if (cllm_err_ != cudaSuccess) ::cudallm::throw_cuda(cllm_err_, #expr, __FILE__, __LINE__); \
    } while (0)

// Internal invariant / launch precondition (maps to CUDALLM_ERR_INTERNAL unless the text says CUDA).
#define CLLM_CHECK(cond, msg)                          \
    do {                                               \
        if (!(cond)) throw std::runtime_error(msg);    \
    } while (0)

// Caller-visible argument check (maps to CUDALLM_ERR_INVALID_ARG).
#define CLLM_REQUIRE(cond, msg)                        \
    do {                                               \
        if (!(cond)) throw ::cudallm::ArgError(msg);   \
    } while (0)
