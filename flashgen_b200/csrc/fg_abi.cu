// fg_abi.cu — C ABI entry points (include/flashgen_sampler.h).
//
// Host side only validates arguments, computes the shared-memory layout and
// launches; it does no work proportional to batch * vocab, allocates nothing
// and never synchronises the stream.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "fg_internal.h"
#include "fg_kernels.cuh"

namespace {

using fg::host::DevInfo;
using fg::host::device_info;
using fg::host::elem_size;
using fg::host::bits_for;
using fg::host::g_mu;

template <int DT>
int launch_sample(const fg::KParams& P, int smem, int grid, cudaStream_t st, DevInfo* d) {
    auto kern = fg::fg_sample_kernel<DT>;
    if (!d->attr_set[fg::host::K_ROW][DT].load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lk(g_mu);
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, d->smem_optin) != cudaSuccess)
            return FG_EDEVICE;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return FG_EDEVICE;
        d->attr_set[fg::host::K_ROW][DT].store(true, std::memory_order_release);
    }
    kern<<<grid, fg::NTHREADS, smem, st>>>(P);
    return cudaGetLastError() == cudaSuccess ? FG_OK : FG_ELAUNCH;
}

}  // namespace

extern "C" {

int fg_version(void) { return 200; }

const char* fg_strerror(int code) {
    switch (code) {
        case FG_OK: return "ok";
        case FG_EINVAL: return "invalid argument";
        case FG_ELAUNCH: return "kernel launch failed";
        case FG_ENOTSUP: return "shape beyond on-chip limits of this build";
        case FG_EDEVICE: return "device query or configuration failed";
        case FG_ESCRATCH: return "request exceeds the fixed scratch of fg_sample_noalloc";
        default: return "unknown error";
    }
}

}  // extern "C"

namespace {
constexpr int32_t kMaxBatch = 1 << 30;

// Shared-memory layout for P (vocab, pen_possible, hu_cap set), then the
// launch of fg_sample_kernel (fg_sample_candidates). mass_vocab: how many
// elements a row's total mass may sum (0: the row's own vocabulary).
int layout_and_launch(fg::KParams& P, int dtype, DevInfo* d, cudaStream_t st, int64_t mass_vocab = 0) {
    P.id_bits = bits_for(std::max<int64_t>(P.vocab, mass_vocab));
    P.mass_shift = 62 - P.id_bits;
    // two CTAs per SM when one fits in half of the SM's shared memory (with at
    // least four 8 KB stages); otherwise one CTA per SM with a deeper ring
    int chosen = 0, smem = 0, per_sm = 1;
    for (int pass = 0; pass < 2 && chosen == 0; ++pass) {
        const int limit = pass == 0 ? (d->smem_per_sm / 2 - 1024) : d->smem_optin;
        const int min_ns = pass == 0 ? 4 : 2;
        for (int ns = 12; ns >= min_ns; --ns) {
            int off = fg::head_bytes(ns);
            const int ob = off; off += 2 * 8 * fg::NB;
            const int oc = off; off += 2 * 4 * fg::NB;
            off = fg::align_up_i(off, 16);
            const int ok = off; off += 4 * fg::CAND_CAP;
            const int oi = off; off += 4 * fg::CAND_CAP;
            int obm = 0, opf = 0, ocn = 0, osv = 0, osc = 0;
            if (P.pen_possible) {
                off = fg::align_up_i(off, 16); obm = off; off += 4 * P.nwords;
                off = fg::align_up_i(off, 16); opf = off; off += 2 * ((P.nwords + 1) / 2);
                off = fg::align_up_i(off, 16); ocn = off; off += 4 * P.hu_cap;
                off = fg::align_up_i(off, 16); osv = off; off += 4 * P.hu_cap;
                off = fg::align_up_i(off, 16); osc = off; off += 4 * P.hu_cap;
            }
            off = fg::align_up_i(off, 128);
            const int total = off + ns * fg::TILE_BYTES;
            if (total <= limit) {
                chosen = ns; smem = total; per_sm = pass == 0 ? 2 : 1;
                P.off_bins = ob; P.off_cnts = oc; P.off_ckey = ok; P.off_cid = oi;
                P.off_bitmap = obm; P.off_prefix = opf; P.off_counts = ocn; P.off_sval = osv; P.off_scol = osc;
                P.off_ring = off;
                break;
            }
        }
    }
    if (chosen == 0) return FG_ENOTSUP;
    P.nstage = chosen;
    P.off_ctl = fg::ctl_offset(chosen);
    const int grid = std::min(P.batch, d->sms * per_sm);
    switch (dtype) {
        case FG_DTYPE_F32: return launch_sample<FG_DTYPE_F32>(P, smem, grid, st, d);
        case FG_DTYPE_F16: return launch_sample<FG_DTYPE_F16>(P, smem, grid, st, d);
        default: return launch_sample<FG_DTYPE_BF16>(P, smem, grid, st, d);
    }
}

// Cluster path mode (fg_cluster.cu): 0 off, 1 automatic, 2 always;
// process-wide, read once per call.
std::atomic<int> g_cluster_mode{1};

// fg_sample's launch; the candidate outputs are non-null only for
// fg_sample_candidates.
int sample_launch(const FgSampleArgs* a, void* stream, float* cvals, int32_t* cids, int32_t* ccount, int32_t cmax) {
    if (a == nullptr) return FG_EINVAL;
    const int esz = elem_size(a->dtype);
    if (esz == 0 || a->logits == nullptr || a->batch < 0 || a->vocab < 1) return FG_EINVAL;
    if (a->row_stride < a->vocab) return FG_EINVAL;
    if ((reinterpret_cast<uintptr_t>(a->logits) % esz) != 0) return FG_EINVAL;
    if (a->temperature == nullptr || a->top_p == nullptr || a->top_k == nullptr || a->uniforms == nullptr ||
        a->out_ids == nullptr || a->workspace == nullptr)
        return FG_EINVAL;
    if (a->workspace_bytes < (size_t)FG_SAMPLE_WORKSPACE_MIN_BYTES) return FG_EINVAL;
    if ((a->hist_ids == nullptr) != (a->hist_offsets == nullptr)) return FG_EINVAL;
    if (a->vocab_offset < 0) return FG_EINVAL;
    const int64_t vtot = a->vocab_total > 0 ? a->vocab_total : a->vocab;
    if (vtot < a->vocab_offset + a->vocab) return FG_EINVAL;
    if (a->vocab > (1 << 28)) return FG_ENOTSUP;
    // the row queue's 32-bit counter runs to about 2 * batch plus one claim per CTA
    if (a->batch > kMaxBatch) return FG_ENOTSUP;
    if (a->batch == 0) return FG_OK;

    DevInfo* d = nullptr;
    int rc = device_info(&d);
    if (rc != FG_OK) return rc;

    fg::KParams P{};
    P.cand_vals = cvals; P.cand_ids = cids; P.cand_count = ccount; P.cand_max = cmax;
    P.logits = a->logits; P.row_stride = a->row_stride; P.batch = a->batch; P.vocab = a->vocab;
    P.vocab_offset = a->vocab_offset; P.vocab_total = vtot;
    P.hist_ids = a->hist_ids; P.hist_offsets = a->hist_offsets;
    P.temperature = a->temperature; P.top_p = a->top_p; P.top_k = a->top_k;
    P.rep = a->repetition_penalty; P.pres = a->presence_penalty; P.freq = a->frequency_penalty;
    P.greedy = a->greedy; P.uniforms = a->uniforms;
    P.out_ids = a->out_ids; P.out_status = a->out_status; P.out_probs = a->out_probs;
    P.ws = reinterpret_cast<fg::Workspace*>(a->workspace);
    P.nwords = (a->vocab + 31) / 32;
    const bool hist = a->hist_offsets != nullptr;
    P.pen_possible = hist && (a->repetition_penalty || a->presence_penalty || a->frequency_penalty);
    if (P.pen_possible) {
        if (a->hist_max_len < 0) return FG_EINVAL;
        P.hu_cap = std::max(1, std::min(a->hist_max_len, a->vocab));
    } else {
        P.hu_cap = 0;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cvals == nullptr) {
        // sampling: small batches (or every batch in mode 2, and calls that
        // want kept-set probabilities) with one cluster per row; otherwise the
        // batch kernel, which hands the rows it cannot decide on chip to the
        // cluster kernel
        const int mode = g_cluster_mode.load(std::memory_order_relaxed);
        int G = fg::host::cluster_size_for(a, d, mode);
        if (G == 0 && a->out_probs != nullptr) G = std::min(4, std::max(1, fg::host::cluster_size_for(a, d, 2)));
        if (G > 0) return fg::host::cluster_launch(a, vtot, true, G, P.pen_possible != 0, P.hu_cap, d, st);
        rc = fg::host::stream_launch(a, vtot, P.pen_possible != 0, P.hu_cap, d, st);
        if (rc != FG_ENOTSUP) return rc;
        G = std::max(1, fg::host::cluster_size_for(a, d, 2) >= 8 ? 8 : fg::host::cluster_size_for(a, d, 2));
        return fg::host::cluster_launch(a, vtot, true, G, P.pen_possible != 0, P.hu_cap, d, st);
    }
    return layout_and_launch(P, a->dtype, d, st);
}
}  // namespace

extern "C" {

int fg_sample(const FgSampleArgs* a, void* stream) {
    return sample_launch(a, stream, nullptr, nullptr, nullptr, 0);
}

int fg_sample_set_split(int mode) {
    if (mode < 0 || mode > 2) return FG_EINVAL;
    g_cluster_mode.store(mode, std::memory_order_relaxed);
    return FG_OK;
}

size_t fg_sample_workspace_size(int32_t batch, int32_t vocab, int32_t dtype, int32_t hist_max_len) {
    if (elem_size(dtype) == 0 || batch < 0 || vocab < 1 || batch > kMaxBatch || hist_max_len < 0) return 0;
    return std::max((size_t)FG_SAMPLE_WORKSPACE_MIN_BYTES,
                    fg::host::stream_workspace_bytes(batch, vocab, hist_max_len, hist_max_len > 0));
}

int fg_sample_candidates(const FgSampleArgs* a, float* vals, int32_t* gids, int32_t* counts, int32_t cand_max,
                         void* stream) {
    if (vals == nullptr || gids == nullptr || counts == nullptr || cand_max < 1) return FG_EINVAL;
    return sample_launch(a, stream, vals, gids, counts, cand_max);
}

// ---------------------------------------------------------------------------
// fg_sample without a caller workspace. Its callers cannot hand the library
// device memory: a C++ engine whose decode loop must not allocate (an
// allocation there can synchronise the device or fail mid-step), and a host
// that binds the library through a plain FFI with no device allocator of its
// own. The row-queue counters live in a file-scope __device__ array instead
// (one per device context). Its address is looked up once per device
// context, on the first call with that device current, which also clears it on
// the call's stream; make that first call before any stream capture. A device
// reset (cudaDeviceReset) ends the context: the next call sees a new context
// id, looks the address up again and clears the array again. Every launch
// leaves the counters zero again. Calls that overlap on the GPU (different
// streams) share the counters and race: serialise them.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = 256;
constexpr int32_t kNoAllocMaxBatch = 1 << 30;   // the queue counter runs to about 2 * batch in 32 bits
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
struct NoAllocSlot {
    unsigned long long ctx_id = 0;   // driver context id the address belongs to (0: none yet)
    void* ptr = nullptr;
};
NoAllocSlot g_noalloc[fg::host::kMaxDevices];
static_assert(sizeof(fg::Workspace) <= kNoAllocScratchBytes, "static scratch smaller than the row-queue counters");

// Unique id of the current driver context (cuCtxGetCurrent + cuCtxGetId,
// reached through the runtime's driver entry points, so the library links no
// libcuda symbol directly). 0 when it cannot be read.
using CtxGetCurrentFn = int (*)(void**);
using CtxGetIdFn = int (*)(void*, unsigned long long*);
unsigned long long current_ctx_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static bool looked_up = false;
    if (!looked_up) {
        void* f0 = nullptr;
        void* f1 = nullptr;
        cudaDriverEntryPointQueryResult q0, q1;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f0, 12000, cudaEnableDefault, &q0) == cudaSuccess &&
            q0 == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(f0);
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f1, 12000, cudaEnableDefault, &q1) == cudaSuccess &&
            q1 == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(f1);
        looked_up = true;
    }
    if (get_current == nullptr || get_id == nullptr) return 0;
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (get_current(&ctx) != 0 || ctx == nullptr) return 0;
    if (get_id(ctx, &id) != 0) return 0;
    return id;
}
}  // namespace

int fg_sample_noalloc(const FgSampleArgs* a, void* stream) {
    if (a == nullptr || a->workspace != nullptr) return FG_EINVAL;
    if (a->batch > kNoAllocMaxBatch) return FG_ESCRATCH;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= fg::host::kMaxDevices) return FG_EDEVICE;
    void* ws = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        NoAllocSlot& slot = g_noalloc[dev];
        unsigned long long id = current_ctx_id();   // 0 before the runtime made a context
        if (slot.ptr == nullptr || id != slot.ctx_id) {
            void* p = nullptr;
            // set-up: the symbol's device address in the current context (the
            // runtime creates or attaches the device's primary context here)
            if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return FG_EDEVICE;
            id = current_ctx_id();
            if (p != slot.ptr || id != slot.ctx_id) {
                if (cudaMemsetAsync(p, 0, kNoAllocScratchBytes, reinterpret_cast<cudaStream_t>(stream)) !=
                    cudaSuccess)
                    return FG_EDEVICE;
            }
            slot.ptr = p;
            slot.ctx_id = id;
        }
        ws = slot.ptr;
    }
    FgSampleArgs b = *a;
    b.workspace = ws;
    b.workspace_bytes = kNoAllocScratchBytes;
    return sample_launch(&b, stream, nullptr, nullptr, nullptr, 0);
}

int fg_argmax(const void* logits, int32_t dtype, int32_t batch, int32_t vocab, int64_t row_stride,
              int64_t* out_ids, void* stream) {
    const int esz = elem_size(dtype);
    if (esz == 0 || logits == nullptr || out_ids == nullptr || batch < 0 || vocab < 1 || row_stride < vocab)
        return FG_EINVAL;
    if ((reinterpret_cast<uintptr_t>(logits) % esz) != 0) return FG_EINVAL;
    if (batch == 0) return FG_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (dtype) {
        case FG_DTYPE_F32: fg::fg_argmax_kernel<FG_DTYPE_F32><<<batch, 256, 0, st>>>(logits, vocab, row_stride, out_ids); break;
        case FG_DTYPE_F16: fg::fg_argmax_kernel<FG_DTYPE_F16><<<batch, 256, 0, st>>>(logits, vocab, row_stride, out_ids); break;
        default: fg::fg_argmax_kernel<FG_DTYPE_BF16><<<batch, 256, 0, st>>>(logits, vocab, row_stride, out_ids); break;
    }
    return cudaGetLastError() == cudaSuccess ? FG_OK : FG_ELAUNCH;
}

int fg_apply_repetition_penalty(void* logits, int32_t dtype, int32_t batch, int32_t vocab, int64_t row_stride,
                                const int32_t* hist_ids, const int64_t* hist_offsets, const float* penalty,
                                void* stream) {
    const int esz = elem_size(dtype);
    if (esz == 0 || logits == nullptr || batch < 0 || vocab < 1 || row_stride < vocab) return FG_EINVAL;
    if ((reinterpret_cast<uintptr_t>(logits) % esz) != 0) return FG_EINVAL;
    if ((hist_ids == nullptr) != (hist_offsets == nullptr)) return FG_EINVAL;
    if (batch == 0 || penalty == nullptr || hist_ids == nullptr) return FG_OK;
    DevInfo* d = nullptr;
    int rc = device_info(&d);
    if (rc != FG_OK) return rc;
    const int smem = 4 * ((vocab + 31) / 32);
    if (smem > d->smem_optin) return FG_ENOTSUP;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    switch (dtype) {
        case FG_DTYPE_F32: {
            auto k = fg::fg_rep_penalty_kernel<FG_DTYPE_F32>;
            if (smem > 48 * 1024) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e == cudaSuccess) k<<<batch, 256, smem, st>>>(logits, vocab, row_stride, hist_ids, hist_offsets, penalty);
            break;
        }
        case FG_DTYPE_F16: {
            auto k = fg::fg_rep_penalty_kernel<FG_DTYPE_F16>;
            if (smem > 48 * 1024) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e == cudaSuccess) k<<<batch, 256, smem, st>>>(logits, vocab, row_stride, hist_ids, hist_offsets, penalty);
            break;
        }
        default: {
            auto k = fg::fg_rep_penalty_kernel<FG_DTYPE_BF16>;
            if (smem > 48 * 1024) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e == cudaSuccess) k<<<batch, 256, smem, st>>>(logits, vocab, row_stride, hist_ids, hist_offsets, penalty);
            break;
        }
    }
    if (e != cudaSuccess) return FG_EDEVICE;
    return cudaGetLastError() == cudaSuccess ? FG_OK : FG_ELAUNCH;
}

}  // extern "C"
