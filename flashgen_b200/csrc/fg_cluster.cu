// fg_cluster.cu — host launch of the cluster kernel (fg_cluster.cuh): one
// thread-block cluster of G CTAs samples one row at a time, each CTA owning a
// slice of the row kept in its shared memory. Used for whole batches that
// would leave most SMs idle with one CTA per row (mode 1: B * G <= SMs with
// G >= 4), for every batch in mode 2, and for the rows the batch kernel
// defers.
#include <algorithm>

#include "fg_internal.h"
#include "fg_cluster.cuh"

namespace fg {
namespace host {

constexpr int kMinSliceChunks = 64;   // 16-byte chunks a CTA should own at least

int cluster_size_for(const FgSampleArgs* a, const DevInfo* d, int mode) {
    const int esz = elem_size(a->dtype);
    const int64_t nch = (int64_t)a->vocab * esz / 16 + 1;
    int gmax = 16;
    while (gmax > 1 && nch / gmax < kMinSliceChunks) gmax >>= 1;
    if (mode == 0) return 0;
    if (mode == 2) return gmax;
    for (int G = gmax; G >= 4; G >>= 1)
        if ((int64_t)a->batch * G <= d->sms) return G;
    return 0;
}

template <int DT>
static int launch_cluster_t(const fg::clus::Params& P, int G, int smem, int nclusters_cap, cudaStream_t st, DevInfo* d) {
    auto kern = fg::clus::cluster_kernel<DT>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(fg::clus::NT, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3((unsigned)G, 1, 1);
    int active = 0;
    {
        // attributes once per device; the co-resident cluster count once per
        // (dtype, cluster size, shared-memory size)
        std::lock_guard<std::mutex> lk(g_mu);
        if (!d->attr_set[K_CLUSTER][DT].load(std::memory_order_acquire)) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, d->smem_optin) != cudaSuccess)
                return FG_EDEVICE;
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
                return FG_EDEVICE;
            d->attr_set[K_CLUSTER][DT].store(true, std::memory_order_release);
        }
        if (d->cl_smem[DT][G] != smem || d->cl_active[DT][G] < 1) {
            if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess || active < 1) return FG_ENOTSUP;
            d->cl_smem[DT][G] = smem;
            d->cl_active[DT][G] = active;
        }
        active = d->cl_active[DT][G];
    }
    const int ncl = std::max(1, std::min(active, nclusters_cap));
    cfg.gridDim = dim3((unsigned)(ncl * G), 1, 1);
    if (cudaLaunchKernelEx(&cfg, kern, P) != cudaSuccess) return FG_ELAUNCH;
    return cudaGetLastError() == cudaSuccess ? FG_OK : FG_ELAUNCH;
}

// all_rows: sample every row; otherwise only the rows whose out_ids holds
// the batch kernel's deferral mark. G: the preferred cluster size; a larger
// one is taken when a CTA's share of the row does not fit its shared memory.
int cluster_launch(const FgSampleArgs* a, int64_t vtot, bool all_rows, int G, bool pen_possible, int hu_cap,
                   DevInfo* d, cudaStream_t st) {
    using namespace fg::clus;
    const int esz = elem_size(a->dtype);
    const int vec = 16 / esz;
    const int64_t nch = (int64_t)a->vocab * esz / 16 + 1;
    Params P{};
    P.logits = a->logits; P.row_stride = a->row_stride; P.batch = a->batch; P.vocab = a->vocab;
    P.vocab_offset = a->vocab_offset; P.vocab_total = vtot;
    P.hist_ids = a->hist_ids; P.hist_offsets = a->hist_offsets;
    P.temperature = a->temperature; P.top_p = a->top_p; P.top_k = a->top_k;
    P.rep = a->repetition_penalty; P.pres = a->presence_penalty; P.freq = a->frequency_penalty;
    P.greedy = a->greedy; P.uniforms = a->uniforms;
    P.out_ids = a->out_ids; P.out_status = a->out_status; P.out_probs = a->out_probs;
    P.ws = reinterpret_cast<unsigned int*>(a->workspace);
    P.all_rows = all_rows ? 1 : 0;
    P.pen_possible = pen_possible ? 1 : 0;
    P.hu_cap = pen_possible ? hu_cap : 0;
    int hs = 64;
    while (hs < 2 * P.hu_cap) hs <<= 1;
    P.hslots = pen_possible ? hs : 0;
    P.mass_shift = 62 - bits_for(a->vocab);
    for (int g = std::max(1, G); g <= GMAX; g <<= 1) {
        const int64_t slice_ch = (nch + g - 1) / g;
        const int64_t ncols = slice_ch * vec + 2 * vec;
        P.swords = pen_possible ? (int)(ncols / 32 + 2) : 0;
        const int64_t cache_words = std::max<int64_t>(ncols, 2 * (int64_t)P.hslots);
        int64_t off = 0;
        P.off_ctl = (int)off; off += align_up((int)sizeof(Ctl), 16);
        P.off_hist = (int)off; off += 4 * hist_words();
        P.off_own = (int)off; off += 4 * own_words(g);
        P.off_full = (int)off; off += 4 * full_words();
        P.off_wloc = (int)off; off += 4 * win_words();
        P.off_wall = (int)off; off += 4 * win_words();
        P.off_bitmap = (int)off; off += align_up(4 * P.swords, 16);
        P.off_hcol = (int)off; off += align_up(4 * P.hu_cap, 16);
        P.off_hval = (int)off; off += align_up(4 * P.hu_cap, 16);
        off = (off + 127) / 128 * 128;
        P.off_cache = (int)off;
        off += 4 * cache_words;
        if (off > d->smem_optin || cache_words > (1 << 28)) continue;
        P.cache_words = (int)cache_words;
        const int smem = (int)off;
        const int cap = all_rows ? std::max(1, a->batch) : 1 << 20;
        switch (a->dtype) {
            case FG_DTYPE_F32: return launch_cluster_t<FG_DTYPE_F32>(P, g, smem, cap, st, d);
            case FG_DTYPE_F16: return launch_cluster_t<FG_DTYPE_F16>(P, g, smem, cap, st, d);
            default: return launch_cluster_t<FG_DTYPE_BF16>(P, g, smem, cap, st, d);
        }
    }
    return FG_ENOTSUP;
}

}  // namespace host
}  // namespace fg
