// platform.h -- errors and checks for the host engine.
// Mirrors src/core/Opure_Platform.h:45-75 (opure::Error, ThrowError, OPURE_CHECK) on Linux,
// plus the mapping from C-ABI status codes to exceptions (OPURE_CUDA_CHECK).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>

#include "opure_cuda.h"

namespace opure {

class Error : public std::runtime_error {
public:
    explicit Error(const std::string &what, opure_status status = OPURE_OK)
        : std::runtime_error(what), status_(status) {}
    opure_status status() const { return status_; }

private:
    opure_status status_;
};

[[noreturn]] inline void ThrowError(const std::string &what, opure_status s = OPURE_OK) {
    throw Error(what, s);
}

}  // namespace opure

#define OPURE_CHECK(cond, msg)                                   \
    do {                                                         \
        if (!(cond)) ::opure::ThrowError(std::string(msg));      \
    } while (0)

// Every call into libopure_cuda goes through this: a non-OK status becomes an
// opure::Error carrying the status (the reference throws on HRESULT failures the
// same way, Opure_Dx12.cpp:53-81).
#define OPURE_CUDA_CHECK(expr)                                                        \
    do {                                                                              \
        const opure_status _s = (expr);                                               \
        if (_s != OPURE_OK)                                                           \
            ::opure::ThrowError(std::string(#expr) + ": " + opure_strerror(_s), _s);   \
    } while (0)
