// fg_bindings.cpp — the PyBind11 module `flashgen_b200._C`: a thin Python
// binding of the C ABI (include/flashgen_sampler.h), the counterpart of the
// reference's `_C` extension (csrc/bindings/flashgen_bindings.cpp:89, which
// binds SamplingParams at :153-162 and releases the GIL around engine calls at
// :235-238).
//
// Device buffers cross as plain integers (device pointers, e.g. a torch
// tensor's data_ptr()) and streams as the cudaStream_t value (0: the legacy
// default stream), so the module needs neither torch nor the CUDA headers.
// Every call releases the GIL; a non-zero status raises RuntimeError with
// fg_strerror's text, the reference's error behaviour on the Python side.
#include <cstdint>
#include <string>
#include <vector>

#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "../../../include/flashgen_sampler.h"

namespace py = pybind11;

namespace {

// The reference's C++ SamplingParams (csrc/include/request.hpp:14-22), with
// the presence and frequency penalties of the sampler added.
struct SamplingParams {
    float temperature = 1.0f;
    float top_p = 0.9f;
    int top_k = -1;  // -1 = disabled
    float repetition_penalty = 1.0f;
    float presence_penalty = 0.0f;
    float frequency_penalty = 0.0f;
    bool greedy = false;
    int max_tokens = 128;
    std::vector<int> stop_token_ids = {50256};  // EOS for GPT-2
};

void check(int rc, const char* what) {
    if (rc != FG_OK) throw std::runtime_error(std::string(what) + " failed: " + fg_strerror(rc) + " (code " +
                                              std::to_string(rc) + ")");
}

template <class T>
T* ptr(std::uintptr_t p) {
    return reinterpret_cast<T*>(p);
}

}  // namespace

PYBIND11_MODULE(_C, m) {
    m.doc() = "flashgen_b200 sampler: PyBind11 binding of the sm_100a C ABI (include/flashgen_sampler.h)";

    py::class_<SamplingParams>(m, "SamplingParams")
        .def(py::init<>())
        .def_readwrite("temperature", &SamplingParams::temperature)
        .def_readwrite("top_p", &SamplingParams::top_p)
        .def_readwrite("top_k", &SamplingParams::top_k)
        .def_readwrite("repetition_penalty", &SamplingParams::repetition_penalty)
        .def_readwrite("presence_penalty", &SamplingParams::presence_penalty)
        .def_readwrite("frequency_penalty", &SamplingParams::frequency_penalty)
        .def_readwrite("greedy", &SamplingParams::greedy)
        .def_readwrite("max_tokens", &SamplingParams::max_tokens)
        .def_readwrite("stop_token_ids", &SamplingParams::stop_token_ids);

    m.attr("DTYPE_F32") = (int)FG_DTYPE_F32;
    m.attr("DTYPE_F16") = (int)FG_DTYPE_F16;
    m.attr("DTYPE_BF16") = (int)FG_DTYPE_BF16;
    m.attr("ROW_ERROR_MASK") = (int)FG_ROW_ERROR_MASK;

    m.def("pack_params",
          [](const std::vector<SamplingParams>& ps) {
              // the structure-of-arrays host vectors fg_sample's per-row
              // parameters are copied from
              const size_t n = ps.size();
              std::vector<float> t(n), p(n), rep(n), pres(n), freq(n);
              std::vector<int32_t> k(n);
              std::vector<uint8_t> g(n);
              for (size_t i = 0; i < n; ++i) {
                  t[i] = ps[i].temperature; p[i] = ps[i].top_p; k[i] = ps[i].top_k;
                  rep[i] = ps[i].repetition_penalty; pres[i] = ps[i].presence_penalty;
                  freq[i] = ps[i].frequency_penalty; g[i] = ps[i].greedy ? 1 : 0;
              }
              return py::make_tuple(t, p, k, rep, pres, freq, g);
          },
          py::arg("params"),
          "Per-row SamplingParams -> (temperature, top_p, top_k, repetition, presence, frequency, greedy) lists");

    m.def("sample",
          [](std::uintptr_t logits, int dtype, int32_t batch, int32_t vocab, int64_t row_stride,
             std::uintptr_t temperature, std::uintptr_t top_p, std::uintptr_t top_k, std::uintptr_t uniforms,
             std::uintptr_t out_ids, std::uintptr_t status, std::uintptr_t repetition_penalty,
             std::uintptr_t presence_penalty, std::uintptr_t frequency_penalty, std::uintptr_t greedy,
             std::uintptr_t hist_ids, std::uintptr_t hist_offsets, int32_t hist_max_len, std::uintptr_t workspace,
             size_t workspace_bytes, std::uintptr_t stream) {
              FgSampleArgs a{};
              a.logits = ptr<const void>(logits);
              a.dtype = dtype;
              a.batch = batch;
              a.vocab = vocab;
              a.row_stride = row_stride > 0 ? row_stride : vocab;
              a.hist_ids = ptr<const int32_t>(hist_ids);
              a.hist_offsets = ptr<const int64_t>(hist_offsets);
              a.hist_max_len = hist_max_len;
              a.temperature = ptr<const float>(temperature);
              a.top_p = ptr<const float>(top_p);
              a.top_k = ptr<const int32_t>(top_k);
              a.repetition_penalty = ptr<const float>(repetition_penalty);
              a.presence_penalty = ptr<const float>(presence_penalty);
              a.frequency_penalty = ptr<const float>(frequency_penalty);
              a.greedy = ptr<const uint8_t>(greedy);
              a.uniforms = ptr<const float>(uniforms);
              a.out_ids = ptr<int64_t>(out_ids);
              a.out_status = ptr<int32_t>(status);
              a.workspace = ptr<void>(workspace);
              a.workspace_bytes = workspace_bytes;
              int rc;
              {
                  py::gil_scoped_release release;
                  rc = fg_sample(&a, ptr<void>(stream));
              }
              check(rc, "fg_sample");
          },
          py::arg("logits"), py::arg("dtype"), py::arg("batch"), py::arg("vocab"), py::arg("row_stride") = 0,
          py::arg("temperature"), py::arg("top_p"), py::arg("top_k"), py::arg("uniforms"), py::arg("out_ids"),
          py::arg("status") = 0, py::arg("repetition_penalty") = 0, py::arg("presence_penalty") = 0,
          py::arg("frequency_penalty") = 0, py::arg("greedy") = 0, py::arg("hist_ids") = 0,
          py::arg("hist_offsets") = 0, py::arg("hist_max_len") = 0, py::arg("workspace") = 0,
          py::arg("workspace_bytes") = 0, py::arg("stream") = 0,
          "fg_sample on device buffers (integers: device pointers; 0: absent). Raises RuntimeError on an error code.");

    m.def("workspace_size",
          [](int32_t batch, int32_t vocab, int32_t dtype, int32_t hist_max_len) {
              return fg_sample_workspace_size(batch, vocab, dtype, hist_max_len);
          },
          py::arg("batch"), py::arg("vocab"), py::arg("dtype"), py::arg("hist_max_len") = 0);

    m.def("argmax",
          [](std::uintptr_t logits, int dtype, int32_t batch, int32_t vocab, int64_t row_stride,
             std::uintptr_t out_ids, std::uintptr_t stream) {
              int rc;
              {
                  py::gil_scoped_release release;
                  rc = fg_argmax(ptr<const void>(logits), dtype, batch, vocab, row_stride > 0 ? row_stride : vocab,
                                 ptr<int64_t>(out_ids), ptr<void>(stream));
              }
              check(rc, "fg_argmax");
          },
          py::arg("logits"), py::arg("dtype"), py::arg("batch"), py::arg("vocab"), py::arg("row_stride") = 0,
          py::arg("out_ids"), py::arg("stream") = 0);

    m.def("apply_repetition_penalty",
          [](std::uintptr_t logits, int dtype, int32_t batch, int32_t vocab, int64_t row_stride,
             std::uintptr_t hist_ids, std::uintptr_t hist_offsets, std::uintptr_t penalty, std::uintptr_t stream) {
              int rc;
              {
                  py::gil_scoped_release release;
                  rc = fg_apply_repetition_penalty(ptr<void>(logits), dtype, batch, vocab,
                                                   row_stride > 0 ? row_stride : vocab, ptr<const int32_t>(hist_ids),
                                                   ptr<const int64_t>(hist_offsets), ptr<const float>(penalty),
                                                   ptr<void>(stream));
              }
              check(rc, "fg_apply_repetition_penalty");
          },
          py::arg("logits"), py::arg("dtype"), py::arg("batch"), py::arg("vocab"), py::arg("row_stride") = 0,
          py::arg("hist_ids"), py::arg("hist_offsets"), py::arg("penalty"), py::arg("stream") = 0);

    m.def("version", []() { return fg_version(); });
    m.def("strerror", [](int code) { return std::string(fg_strerror(code)); });
}
