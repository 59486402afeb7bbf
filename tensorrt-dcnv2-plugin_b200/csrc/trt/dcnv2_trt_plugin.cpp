// dcnv2_trt_plugin.cpp — TensorRT 10 IPluginV3 adapter over the libdcnv2 C ABI.
//
// Registers a creator named "DCNv2", version "1", namespace "" — the identity of the reference
// plugin (src/dcn_plugin.cpp:22-23, 199, 238-244) — so that engines and ONNX graphs that use the
// `dcn::DCNv2` node bind to this library instead. Every decision (attribute parsing and defaults,
// output shape and type, format combinations, workspace size, the forward itself) is delegated to
// the dcnv2_plugin_* functions of include/dcnv2.h; this file only converts TensorRT types.
//
// Built only when TensorRT headers are available (Makefile: TRT_INCLUDE_DIR=/path/to/include),
// into the same libdcnv2.so; loading the library with dlopen / ctypes.CDLL registers the creator
// (REGISTER_TENSORRT_PLUGIN), exactly as the reference's libdcnv2.so did, and the library also
// exports getCreators / setLoggerFinder for IPluginRegistry::loadLibrary.

#include <NvInfer.h>
#include <NvInferRuntime.h>

#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../../include/dcnv2.h"

namespace dcnv2_trt {

using namespace nvinfer1;

// PluginTensorDesc -> dcnv2_tensor_desc (type values are shared with nvinfer1::DataType).
dcnv2_tensor_desc to_desc(PluginTensorDesc const& d) {
  dcnv2_tensor_desc r;
  std::memset(&r, 0, sizeof(r));
  r.nb_dims = d.dims.nbDims;
  for (int i = 0; i < d.dims.nbDims && i < 8; ++i) r.d[i] = d.dims.d[i];
  r.type = static_cast<int32_t>(d.type);
  r.format = static_cast<int32_t>(d.format);
  r.scale = d.scale;
  return r;
}

class Plugin final : public IPluginV3,
                     public IPluginV3OneCore,
                     public IPluginV3OneBuild,
                     public IPluginV3OneRuntime {
 public:
  explicit Plugin(dcnv2_plugin* impl) : impl_(impl) { refresh_fields(); }
  ~Plugin() override { dcnv2_plugin_destroy(impl_); }
  Plugin(Plugin const&) = delete;
  Plugin& operator=(Plugin const&) = delete;

  // ---- IPluginV3
  IPluginCapability* getCapabilityInterface(PluginCapabilityType type) noexcept override {
    if (type == PluginCapabilityType::kCORE) return static_cast<IPluginV3OneCore*>(this);
    if (type == PluginCapabilityType::kBUILD) return static_cast<IPluginV3OneBuild*>(this);
    if (type == PluginCapabilityType::kRUNTIME) return static_cast<IPluginV3OneRuntime*>(this);
    return nullptr;
  }
  IPluginV3* clone() noexcept override {
    dcnv2_plugin* c = dcnv2_plugin_clone(impl_);
    return c ? new (std::nothrow) Plugin(c) : nullptr;
  }

  // ---- IPluginV3OneCore
  AsciiChar const* getPluginName() const noexcept override { return dcnv2_plugin_name(); }
  AsciiChar const* getPluginVersion() const noexcept override { return dcnv2_plugin_version(); }
  AsciiChar const* getPluginNamespace() const noexcept override { return dcnv2_plugin_namespace(); }

  // ---- IPluginV3OneBuild
  int32_t getNbOutputs() const noexcept override { return dcnv2_plugin_nb_outputs(impl_); }

  int32_t getOutputDataTypes(DataType* out, int32_t nb_out, DataType const* in,
                             int32_t nb_in) const noexcept override {
    if (nb_out != 1 || nb_in < 1) return -1;
    out[0] = static_cast<DataType>(dcnv2_plugin_output_dtype(impl_, static_cast<int32_t>(in[0])));
    return 0;
  }

  // y = [N, O, Ho, Wo] with Ho = floor((H + 2p - d(K-1) - 1) / s) + 1 as shape expressions.
  int32_t getOutputShapes(DimsExprs const* in, int32_t nb_in, DimsExprs const*, int32_t,
                          DimsExprs* out, int32_t nb_out, IExprBuilder& eb) noexcept override {
    if (nb_in != 5 || nb_out != 1 || in[0].nbDims != 4 || in[3].nbDims != 4) return -1;
    int32_t f[5];
    dcnv2_plugin_serialize(impl_, nullptr, f);  // stride, padding, dilation, kernel, groups
    const int32_t s = f[0], p = f[1], d = f[2], k = f[3];
    auto extent = [&](IDimensionExpr const* len) {
      // len + 2p - d(k-1) - 1, floor-divided by s, + 1
      IDimensionExpr const* num = eb.operation(DimensionOperation::kSUM, *len,
                                               *eb.constant(2 * p - d * (k - 1) - 1));
      IDimensionExpr const* q = eb.operation(DimensionOperation::kFLOOR_DIV, *num, *eb.constant(s));
      return eb.operation(DimensionOperation::kSUM, *q, *eb.constant(1));
    };
    out[0].nbDims = 4;
    out[0].d[0] = in[0].d[0];
    out[0].d[1] = in[3].d[0];
    out[0].d[2] = extent(in[0].d[2]);
    out[0].d[3] = extent(in[0].d[3]);
    return 0;
  }

  bool supportsFormatCombination(int32_t pos, DynamicPluginTensorDesc const* io, int32_t nb_in,
                                 int32_t nb_out) noexcept override {
    std::vector<dcnv2_tensor_desc> v(static_cast<size_t>(nb_in + nb_out));
    for (int32_t i = 0; i < nb_in + nb_out; ++i) v[i] = to_desc(io[i].desc);
    return dcnv2_plugin_supports_format(impl_, pos, v.data(), nb_in, nb_out) != 0;
  }

  int32_t configurePlugin(DynamicPluginTensorDesc const*, int32_t, DynamicPluginTensorDesc const*,
                          int32_t) noexcept override {
    return 0;
  }

  // Sized for the largest shapes of the optimisation profile (the need grows with N, H, W).
  size_t getWorkspaceSize(DynamicPluginTensorDesc const* in, int32_t nb_in,
                          DynamicPluginTensorDesc const* out, int32_t nb_out) const noexcept override {
    std::vector<dcnv2_tensor_desc> vi(static_cast<size_t>(nb_in)), vo(static_cast<size_t>(nb_out));
    for (int32_t i = 0; i < nb_in; ++i) {
      vi[i] = to_desc(in[i].desc);
      for (int j = 0; j < in[i].max.nbDims && j < 8; ++j) vi[i].d[j] = in[i].max.d[j];
    }
    for (int32_t i = 0; i < nb_out; ++i) {
      vo[i] = to_desc(out[i].desc);
      for (int j = 0; j < out[i].max.nbDims && j < 8; ++j) vo[i].d[j] = out[i].max.d[j];
    }
    return dcnv2_plugin_workspace_size(impl_, vi.data(), nb_in, vo.data(), nb_out);
  }

  // ---- IPluginV3OneRuntime
  int32_t onShapeChange(PluginTensorDesc const*, int32_t, PluginTensorDesc const*,
                        int32_t) noexcept override {
    return 0;
  }

  int32_t enqueue(PluginTensorDesc const* in_desc, PluginTensorDesc const* out_desc,
                  void const* const* inputs, void* const* outputs, void* workspace,
                  cudaStream_t stream) noexcept override {
    dcnv2_tensor_desc vi[5], vo[1];
    for (int i = 0; i < 5; ++i) vi[i] = to_desc(in_desc[i]);
    vo[0] = to_desc(out_desc[0]);
    // the exact need of these shapes; TensorRT provides at least the profile maximum
    const size_t ws = dcnv2_plugin_workspace_size(impl_, vi, 5, vo, 1);
    return dcnv2_plugin_enqueue(impl_, vi, vo, inputs, outputs, workspace, ws,
                                static_cast<dcnv2_stream_t>(stream));
  }

  IPluginV3* attachToContext(IPluginResourceContext*) noexcept override { return clone(); }

  PluginFieldCollection const* getFieldsToSerialize() noexcept override {
    refresh_fields();
    return &fc_;
  }

 private:
  void refresh_fields() {
    dcnv2_plugin_serialize(impl_, names_, values_);
    fields_.clear();
    for (int i = 0; i < 5; ++i)
      fields_.emplace_back(names_[i], &values_[i], PluginFieldType::kINT32, 1);
    fc_.nbFields = static_cast<int32_t>(fields_.size());
    fc_.fields = fields_.data();
  }

  dcnv2_plugin* impl_;
  const char* names_[5] = {};
  int32_t values_[5] = {};
  std::vector<PluginField> fields_;
  PluginFieldCollection fc_{};
};

class Creator final : public IPluginCreatorV3One {
 public:
  Creator() {
    const char* const* names = nullptr;
    const int32_t n = dcnv2_plugin_field_names(&names);
    for (int32_t i = 0; i < n; ++i)
      attrs_.emplace_back(names[i], nullptr, PluginFieldType::kINT32, 1);
    fc_.nbFields = static_cast<int32_t>(attrs_.size());
    fc_.fields = attrs_.data();
  }

  IPluginV3* createPlugin(AsciiChar const*, PluginFieldCollection const* fc,
                          TensorRTPhase) noexcept override {
    std::vector<const char*> names;
    std::vector<const int32_t*> values;
    if (fc) {
      for (int32_t i = 0; i < fc->nbFields; ++i) {
        const PluginField& f = fc->fields[i];
        if (f.type != PluginFieldType::kINT32 || f.length < 1) continue;  // INT32 attributes only
        names.push_back(f.name);
        values.push_back(static_cast<const int32_t*>(f.data));
      }
    }
    dcnv2_plugin* p = dcnv2_plugin_create(names.data(), values.data(),
                                          static_cast<int32_t>(names.size()));
    return p ? new (std::nothrow) Plugin(p) : nullptr;
  }

  PluginFieldCollection const* getFieldNames() noexcept override { return &fc_; }
  AsciiChar const* getPluginName() const noexcept override { return dcnv2_plugin_name(); }
  AsciiChar const* getPluginVersion() const noexcept override { return dcnv2_plugin_version(); }
  AsciiChar const* getPluginNamespace() const noexcept override { return dcnv2_plugin_namespace(); }

 private:
  std::vector<PluginField> attrs_;
  PluginFieldCollection fc_{};
};

}  // namespace dcnv2_trt

REGISTER_TENSORRT_PLUGIN(dcnv2_trt::Creator);

// Plugin-library entry points of TensorRT 10 (IPluginRegistry::loadLibrary, trtexec
// --dynamicPlugins): the library's creators, and the logger finder TensorRT hands over before
// asking for them (this library logs nothing itself, so it is only accepted).
extern "C" {
__attribute__((visibility("default"))) void setLoggerFinder(nvinfer1::ILoggerFinder* finder) {
  (void)finder;
}
__attribute__((visibility("default"))) nvinfer1::IPluginCreatorInterface* const* getCreators(
    int32_t& nbCreators) {
  static dcnv2_trt::Creator creator;
  static nvinfer1::IPluginCreatorInterface* const creators[] = {&creator};
  nbCreators = 1;
  return creators;
}
}
