// fg_stream.cu — host launch of the batch path (fg_stream.cuh): K1 (history
// lists, when the call has penalties), K2 (the stream), K3 (decisions), K4
// (16-bit rows whose cut or draw lies below the candidates), then the cluster
// kernel over the rows K3 and K4 defer. All on the caller's stream.
#include <algorithm>

#include "fg_internal.h"
#include "fg_stream.cuh"

namespace fg {
namespace host {

namespace {

constexpr int kCap = 3072;            // candidate entries (shared memory and row block)
constexpr int kMinStages = 3;

template <class K>
int set_smem_attr(K kern, DevInfo* d, int family, int dt) {
    if (d->attr_set[family][dt].load(std::memory_order_acquire)) return FG_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    if (d->attr_set[family][dt].load(std::memory_order_relaxed)) return FG_OK;
    // the dynamic share of the opt-in limit: what the kernel's static shared memory leaves
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return FG_EDEVICE;
    const int dyn = d->smem_optin - (int)fa.sharedSizeBytes;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) != cudaSuccess)
        return FG_EDEVICE;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
        return FG_EDEVICE;
    d->attr_set[family][dt].store(true, std::memory_order_release);
    return FG_OK;
}

int hu_cap_of(bool pen_possible, int hist_max_len, int vocab) {
    return pen_possible ? std::max(1, std::min(hist_max_len, vocab)) : 0;
}
int hslots_of(int hu_cap) {
    int hs = 64;
    while (hs < 2 * hu_cap) hs <<= 1;
    return hs;
}

template <int DT>
int launch_all(strm::Params& P, int k2_smem, int k2_grid, int k1_smem, int k3_smem, int k4_smem, cudaStream_t st,
               DevInfo* d) {
    int rc;
    if (P.pen_possible) {
        rc = set_smem_attr(strm::prep_kernel<DT>, d, K_PREP, DT);
        if (rc != FG_OK) return rc;
        strm::prep_kernel<DT><<<P.batch, strm::NCT, k1_smem, st>>>(P);
        if (cudaGetLastError() != cudaSuccess) return FG_ELAUNCH;
    }
    rc = set_smem_attr(strm::stream_kernel<DT>, d, K_STREAM, DT);
    if (rc != FG_OK) return rc;
    strm::stream_kernel<DT><<<k2_grid, strm::NTH, k2_smem, st>>>(P);
    if (cudaGetLastError() != cudaSuccess) return FG_ELAUNCH;
    rc = set_smem_attr(strm::decide_kernel<DT>, d, K_DECIDE, DT);
    if (rc != FG_OK) return rc;
    const int k3_grid = std::max(1, std::min(P.batch, d->sms * 8));
    strm::decide_kernel<DT><<<k3_grid, strm::NCT, k3_smem, st>>>(P);
    if (cudaGetLastError() != cudaSuccess) return FG_ELAUNCH;
    if constexpr (DT != FG_DTYPE_F32) {
        // K4: 16-bit rows whose top-p cut or draw lies below the candidates
        rc = set_smem_attr(strm::deep_kernel<DT>, d, K_DEEP, DT);
        if (rc != FG_OK) return rc;
        strm::deep_kernel<DT><<<k3_grid, strm::DNT, k4_smem, st>>>(P);
        if (cudaGetLastError() != cudaSuccess) return FG_ELAUNCH;
    } else {
        (void)k4_smem;
    }
    return FG_OK;
}

}  // namespace

size_t stream_workspace_bytes(int64_t batch, int vocab, int hist_max_len, bool pen_possible) {
    const int hu = hu_cap_of(pen_possible, hist_max_len, vocab);
    return 256 + (size_t)batch * (size_t)strm::wrow_bytes(hu, kCap);
}

// The batch path over every row, then the cluster kernel over the rows it
// deferred. FG_ENOTSUP when the layouts or the workspace cannot hold this
// call (the caller then samples every row with the cluster kernel).
int stream_launch(const FgSampleArgs* a, int64_t vtot, bool pen_possible, int hu_cap, DevInfo* d, cudaStream_t st) {
    strm::Params P{};
    P.logits = a->logits; P.row_stride = a->row_stride; P.batch = a->batch; P.vocab = a->vocab;
    P.vocab_offset = a->vocab_offset; P.vocab_total = vtot;
    P.hist_ids = a->hist_ids; P.hist_offsets = a->hist_offsets;
    P.temperature = a->temperature; P.top_p = a->top_p; P.top_k = a->top_k;
    P.rep = a->repetition_penalty; P.pres = a->presence_penalty; P.freq = a->frequency_penalty;
    P.greedy = a->greedy; P.uniforms = a->uniforms;
    P.out_ids = a->out_ids; P.out_status = a->out_status;
    P.ws = reinterpret_cast<unsigned int*>(a->workspace);
    P.pen_possible = pen_possible ? 1 : 0;
    P.hu_cap = pen_possible ? hu_cap : 0;
    P.hcap4 = (P.hu_cap + 3) / 4 * 4;
    P.hslots = pen_possible ? hslots_of(P.hu_cap) : 0;
    P.nwords = pen_possible ? (a->vocab + 31) / 32 : 0;
    P.mass_shift = 62 - bits_for(a->vocab);
    P.cap = kCap;
    P.k_fast = kCap / 2;
    P.k_nuc = kCap / 3;
    // the workspace holds a block per row after the counters
    P.wrow_bytes = strm::wrow_bytes(P.hu_cap, P.cap);
    const size_t need = 256 + (size_t)a->batch * (size_t)P.wrow_bytes;
    if (a->workspace_bytes < need) return FG_ENOTSUP;
    P.wrow = reinterpret_cast<uint8_t*>(a->workspace) + 256;
    // K2: two CTAs per SM, the deepest ring that fits
    int off = 0;
    const int per_sm = 2;
    const int limit = std::min(d->smem_optin, d->smem_per_sm / per_sm - 1024);
    int ns = 0, fixed = 0;
    for (int n = 16; n >= kMinStages; --n) {
        off = align_up(strm::bar_bytes(n), 16);
        P.off_ctl = off; off += align_up((int)sizeof(strm::Ctl), 16);
        P.off_bins = off; off += 3 * strm::NB * 4;
        P.off_ckey = off; off += 4 * P.cap;
        P.off_ccol = off; off += 4 * P.cap;
        P.off_hbm = off; off += align_up(4 * (P.nwords + 1), 16);   // history column bitmap
        off = align_up(off, 128);
        P.off_ring = off;
        if (off + n * strm::TILE <= limit) { ns = n; fixed = off; break; }
    }
    if (ns == 0) return FG_ENOTSUP;
    P.nstage = ns;
    const int k2_smem = fixed + ns * strm::TILE;
    const int k3_smem = P.off_hbm;                   // control, bins and the candidate buffer
    P.off_cnt = align_up(P.off_hbm + 4 * (P.nwords + 1), 16);
    P.off_tsum = P.off_cnt + 4 * strm::NBIN;
    P.off_hl = P.off_tsum + 8 * (strm::NCT + strm::SLOTS);
    const int k4_smem = P.off_hl + 8 * strm::HL_MAX;
    if (k4_smem + strm::kDeepStaticSmem > d->smem_optin) return FG_ENOTSUP;
    const int k1_smem = align_up(P.off_ctl + (int)sizeof(strm::Ctl), 16) + 8 * P.hslots + 4 * (P.hslots / 2);
    if (pen_possible && k1_smem > d->smem_optin) return FG_ENOTSUP;
    const int k2_grid = std::max(1, std::min(a->batch, d->sms * per_sm));
    int rc;
    switch (a->dtype) {
        case FG_DTYPE_F32: rc = launch_all<FG_DTYPE_F32>(P, k2_smem, k2_grid, k1_smem, k3_smem, k4_smem, st, d); break;
        case FG_DTYPE_F16: rc = launch_all<FG_DTYPE_F16>(P, k2_smem, k2_grid, k1_smem, k3_smem, k4_smem, st, d); break;
        default: rc = launch_all<FG_DTYPE_BF16>(P, k2_smem, k2_grid, k1_smem, k3_smem, k4_smem, st, d); break;
    }
    if (rc != FG_OK) return rc;
    const int gm = cluster_size_for(a, d, 2);
    const int G = std::max(1, gm >= 8 ? 8 : gm);
    return cluster_launch(a, vtot, false, G, pen_possible, hu_cap, d, st);
}

}  // namespace host
}  // namespace fg
