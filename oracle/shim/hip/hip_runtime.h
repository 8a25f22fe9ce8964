/* TEST INFRASTRUCTURE ONLY.  Host-memory stand-in for the few HIP runtime
 * calls made by the reference's src/runner/buffers.cpp, so that file and
 * src/runner/cpu_ref.cpp compile unmodified with g++ into oracle/_ref.
 * "Device" buffers become plain host allocations; nothing here runs a GPU. */
#pragma once
#include <cstddef>
#include <cstdlib>
#include <cstring>

typedef int hipError_t;
typedef void* hipStream_t;
#define hipSuccess 0
enum hipMemcpyKind { hipMemcpyHostToHost, hipMemcpyHostToDevice, hipMemcpyDeviceToHost,
                     hipMemcpyDeviceToDevice, hipMemcpyDefault };

inline hipError_t hipMalloc(void** p, size_t n) {
    *p = std::malloc(n ? n : 1);
    return *p ? hipSuccess : 2;
}
inline hipError_t hipFree(void* p) { std::free(p); return hipSuccess; }
inline hipError_t hipMemcpy(void* dst, const void* src, size_t n, hipMemcpyKind) {
    std::memcpy(dst, src, n);
    return hipSuccess;
}
inline hipError_t hipMemset(void* dst, int v, size_t n) { std::memset(dst, v, n); return hipSuccess; }
inline const char* hipGetErrorString(hipError_t) { return "host shim error"; }
