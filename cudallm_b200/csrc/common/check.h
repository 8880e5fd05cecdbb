// Host-side errors. Every failure this library raises is a cudallm::Error that carries the C-ABI return
// code it maps to (include/cudallm.h: 1 INVALID_ARG, 2 IO, 3 FORMAT, 4 CUDA, 5 STATE, 6 INTERNAL), so the
// ABI layer reads the code off the exception instead of classifying it. The subclasses only fix the code.
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace cudallm {

enum class Status : int { OK = 0, INVALID_ARG = 1, IO = 2, FORMAT = 3, CUDA = 4, STATE = 5, INTERNAL = 6 };

class Error : public std::runtime_error {
public:
    Error(Status s, const std::string& msg) : std::runtime_error(msg), status_(s) {}
    Status status() const noexcept { return status_; }

private:
    Status status_;
};

// A caller-supplied argument or option is invalid (nothing was done).
struct ArgError : Error {
    explicit ArgError(const std::string& m) : Error(Status::INVALID_ARG, m) {}
};
// A file cannot be opened or read.
struct IoError : Error {
    explicit IoError(const std::string& m) : Error(Status::IO, m) {}
};
// A file's header or tensor table breaks the .cudallm format rules.
struct FormatError : Error {
    explicit FormatError(const std::string& m) : Error(Status::FORMAT, m) {}
};
// The engine cannot take the request in its current state (full sequence, failed device wait, ...).
struct StateError : Error {
    explicit StateError(const std::string& m) : Error(Status::STATE, m) {}
};
// A CUDA runtime call failed; the message names the call and always contains "CUDA".
struct CudaError : Error {
    explicit CudaError(const std::string& m) : Error(Status::CUDA, m) {}
};
// A broken internal invariant (a bug, not a caller mistake).
struct InternalError : Error {
    explicit InternalError(const std::string& m) : Error(Status::INTERNAL, m) {}
};

[[noreturn]] inline void throw_cuda(cudaError_t err, const char* expr, const char* file, int line) {
    throw CudaError(std::string("CUDA error ") + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ") from " + expr +
                    " at " + file + ":" + std::to_string(line));
}

}  // namespace cudallm

#define CLLM_CUDA(expr)                                                                            \
    do {                                                                                           \
        const cudaError_t cllm_err_ = (expr);                                                      \
        if (cllm_err_ != cudaSuccess) ::cudallm::throw_cuda(cllm_err_, #expr, __FILE__, __LINE__); \
    } while (0)

// Internal invariant or launch precondition (INTERNAL).
#define CLLM_CHECK(cond, msg)                                  \
    do {                                                       \
        if (!(cond)) throw ::cudallm::InternalError(msg);      \
    } while (0)

// Caller-visible argument check (INVALID_ARG).
#define CLLM_REQUIRE(cond, msg)                                \
    do {                                                       \
        if (!(cond)) throw ::cudallm::ArgError(msg);           \
    } while (0)
