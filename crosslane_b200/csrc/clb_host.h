// Host-side helpers shared by the library's C-ABI translation units: errors carry a
// CLB_E_* code and a message, and `guarded` turns them (and allocation failures) into the
// status + clb_error_v1 convention of every entry point.
#pragma once
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <stdexcept>
#include <string>

#include <cuda_runtime.h>

#include "../../include/crosslane_b200.h"

namespace {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void require(bool ok, int code, const char* fmt, ...) {
    if (ok) return;
    char buf[480];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    throw Error(code, buf);
}

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Error(CLB_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int fail(clb_error_v1* err, int code, const char* msg) {
    if (err) {
        err->code = code;
        std::snprintf(err->message, sizeof err->message, "%s", msg);
    }
    return code;
}

template <class F>
int guarded(clb_error_v1* err, F&& f) {
    try {
        f();
        if (err) {
            err->code = CLB_OK;
            err->message[0] = 0;
        }
        return CLB_OK;
    } catch (const Error& e) {
        return fail(err, e.code, e.what());
    } catch (const std::bad_alloc&) {
        return fail(err, CLB_E_NOMEM, "host allocation failed");
    } catch (const std::exception& e) {
        return fail(err, CLB_E_INVALID, e.what());
    }
}

}  // namespace
