// device_state.cpp -- see device_state.hpp.
#include "device_state.hpp"

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <set>
#include <utility>

namespace uq {

namespace {
std::mutex g_mu;
std::set<std::pair<int, int>> g_done;
std::map<int, int> g_sms;
}  // namespace

bool once_per_device(int family, const std::function<bool()> &set) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_done.count({dev, family})) return true;
    if (!set()) return false;
    g_done.insert({dev, family});
    return true;
}

int current_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_sms.find(dev);
    if (it != g_sms.end()) return it->second;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
    return n;
}

}  // namespace uq
