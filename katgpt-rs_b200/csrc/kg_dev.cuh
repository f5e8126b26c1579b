// kg_dev.cuh — per-device launch state shared by the kernel launchers.
//
// A kernel's dynamic shared-memory limit (cudaFuncAttributeMaxDynamicSharedMemorySize)
// is an attribute of the kernel on one device, and SM counts and occupancy
// are properties of one device. One process may drive several GPUs (one
// context per device, from one or several host threads), so every such value
// is kept per (device, kernel) behind a mutex instead of in a process-wide
// static. The first launch of a kernel on a device is an eager call (decode
// graphs are captured from the second call of a batch shape on), so captures
// only read these tables.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <tuple>
#include <utility>

namespace kg {
namespace dev {

inline int current() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

struct Tables {
    std::mutex mu;
    std::map<std::pair<int, const void *>, size_t> smem;           // (device, kernel) -> limit set
    std::map<std::tuple<int, const void *, int, size_t>, int> occ;  // (device, kernel, threads, smem) -> CTAs/SM
    std::map<int, int> sms;                                         // device -> SM count
};
inline Tables &tables() {
    static Tables t;
    return t;
}

// Raise `fn`'s dynamic shared-memory limit on the current device to at least `bytes`.
inline cudaError_t smem_raw(const void *fn, size_t bytes) {
    const int d = current();
    Tables &t = tables();
    std::lock_guard<std::mutex> lk(t.mu);
    size_t &have = t.smem[{d, fn}];
    if (have >= bytes) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}
template <typename... A>
inline cudaError_t smem(void (*fn)(A...), size_t bytes) {
    return smem_raw(reinterpret_cast<const void *>(fn), bytes);
}

// SM count of the current device.
inline int sm_count() {
    const int d = current();
    Tables &t = tables();
    std::lock_guard<std::mutex> lk(t.mu);
    auto it = t.sms.find(d);
    if (it != t.sms.end()) return it->second;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) n = 148;
    t.sms[d] = n;
    return n;
}

// Resident CTAs per SM of `fn` at (threads, dynamic smem) on the current device (>= 1).
template <typename... A>
inline int occupancy(void (*fn)(A...), int threads, size_t smem_bytes) {
    const void *f = reinterpret_cast<const void *>(fn);
    const int d = current();
    Tables &t = tables();
    std::lock_guard<std::mutex> lk(t.mu);
    auto key = std::make_tuple(d, f, threads, smem_bytes);
    auto it = t.occ.find(key);
    if (it != t.occ.end()) return it->second;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, f, threads, smem_bytes) != cudaSuccess || n < 1) n = 1;
    t.occ[key] = n;
    return n;
}

}  // namespace dev
}  // namespace kg
