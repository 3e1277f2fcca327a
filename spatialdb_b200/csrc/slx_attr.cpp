// slx_attr.cpp -- per-device kernel attributes (see slx_attr.h).
#include "slx_attr.h"

#include <map>
#include <mutex>
#include <utility>

namespace slx {
namespace {
std::mutex g_mu;
std::map<std::pair<const void*, int>, size_t> g_smem;  // (kernel, device) -> limit set there
std::map<int, int> g_sms;                              // device -> SM count
}  // namespace

cudaError_t ensure_smem(const void* func, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_mu);
    size_t& have = g_smem[{func, dev}];
    if (have >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

int device_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_sms.find(dev);
    if (it != g_sms.end()) return it->second;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
    return n;
}

}  // namespace slx
