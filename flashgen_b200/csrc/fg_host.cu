// fg_host.cu — host helpers shared by the library's translation units.
#include "fg_internal.h"

namespace fg {
namespace host {

std::mutex g_mu;

namespace {
DevInfo g_dev[kMaxDevices];
}  // namespace

int device_info(DevInfo** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FG_EDEVICE;
    std::lock_guard<std::mutex> lk(g_mu);
    DevInfo& d = g_dev[dev];
    if (!d.ok) {
        if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return FG_EDEVICE;
        if (cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
            return FG_EDEVICE;
        if (cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess)
            return FG_EDEVICE;
        d.ok = true;
    }
    *out = &d;
    return FG_OK;
}

}  // namespace host
}  // namespace fg
