// fg_internal.h — host-side helpers shared by the library's translation units
// (fg_abi.cu: the C ABI and the per-row kernel; fg_cluster.cu: the cluster
// kernel; fg_stream.cu: the batch kernel). Not part of the public ABI.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>

#include <cuda_runtime.h>

#include "../../include/flashgen_sampler.h"

namespace fg {
namespace host {

struct DevInfo {
    int sms = 0;
    int smem_optin = 0;
    int smem_per_sm = 0;
    // one-time kernel attributes, per kernel family (see the K_* ids) and
    // dtype: read without the lock (acquire), set under it (release)
    std::atomic<bool> attr_set[6][3] = {};
    // cluster kernel: co-resident clusters per (dtype, cluster size) for the
    // shared-memory size it was last queried with
    int cl_smem[3][17] = {};
    int cl_active[3][17] = {};
    bool ok = false;
};
constexpr int kMaxDevices = 64;
enum KernelFamily { K_ROW = 0, K_STREAM = 1, K_CLUSTER = 2, K_PREP = 3, K_DECIDE = 4, K_DEEP = 5 };

// Attributes of the current device (queried once per device, cached).
int device_info(DevInfo** out);
// Serialises the one-time set-up steps of every translation unit.
extern std::mutex g_mu;

inline int elem_size(int dtype) {
    switch (dtype) {
        case FG_DTYPE_F32: return 4;
        case FG_DTYPE_F16: return 2;
        case FG_DTYPE_BF16: return 2;
        default: return 0;
    }
}
inline int bits_for(int64_t v) {  // smallest b >= 1 with v <= 2^b
    int b = 1;
    while ((int64_t(1) << b) < v) ++b;
    return b;
}
inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

// Cluster kernel (fg_cluster.cu): cluster size for a whole batch in `mode`
// (0 when the batch should not take the cluster path), and its launch over
// every row (all_rows) or over the rows the batch kernel deferred.
int cluster_size_for(const FgSampleArgs* a, const DevInfo* d, int mode);
int cluster_launch(const FgSampleArgs* a, int64_t vocab_total, bool all_rows, int G, bool pen_possible, int hu_cap,
                   DevInfo* d, cudaStream_t st);
// Batch kernel (fg_stream.cu) over every row, then the cluster kernel over the
// rows it deferred; FG_ENOTSUP when its shared-memory layout cannot hold the call.
int stream_launch(const FgSampleArgs* a, int64_t vocab_total, bool pen_possible, int hu_cap, DevInfo* d,
                  cudaStream_t st);
// Workspace bytes the batch path needs for this shape (row blocks after the counters).
size_t stream_workspace_bytes(int64_t batch, int vocab, int hist_max_len, bool pen_possible);

}  // namespace host
}  // namespace fg
