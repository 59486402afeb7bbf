// dcnv2_plugin.cpp — the dcn::DCNv2 plugin object (identity, attributes, shape inference,
// precision negotiation, workspace rule, enqueue dispatch, field serialisation) written against
// plain C types, so that a TensorRT IPluginV3 shim (trt/dcnv2_trt_plugin.cpp) and any FFI share
// one implementation. Each function mirrors the reference method named beside it in
// include/dcnv2.h (src/dcn_plugin.cpp of flairziv/tensorrt-dcnv2-plugin).
#include <cstdint>
#include <cstring>
#include <new>

#include "../../include/dcnv2.h"

struct dcnv2_plugin {
  int32_t kernel = 3, stride = 1, padding = 1, dilation = 1, deformable_groups = 1;
};

namespace {
const char* const kFieldNames[5] = {"stride", "padding", "dilation", "kernel",
                                    "deformable_groups"};

bool type_ok(int32_t t) { return t == DCNV2_FLOAT || t == DCNV2_HALF || t == DCNV2_INT8; }

int32_t to_i32(int64_t v) {
  if (v > INT32_MAX || v < INT32_MIN) return -1;
  return static_cast<int32_t>(v);
}
}  // namespace

extern "C" {

const char* dcnv2_plugin_name(void) { return "DCNv2"; }
const char* dcnv2_plugin_version(void) { return "1"; }
const char* dcnv2_plugin_namespace(void) { return ""; }

int32_t dcnv2_plugin_field_names(const char* const** names) {
  if (names) *names = kFieldNames;
  return 5;
}

dcnv2_plugin* dcnv2_plugin_create(const char* const* names, const int32_t* const* values,
                                  int32_t nb_fields) {
  dcnv2_plugin* p = new (std::nothrow) dcnv2_plugin();
  if (!p) return nullptr;
  for (int32_t i = 0; i < nb_fields && names; ++i) {
    const char* nm = names[i];
    if (!nm) continue;
    const int32_t v = (values && values[i]) ? *values[i] : 0;
    if (!std::strcmp(nm, "stride")) p->stride = v;
    else if (!std::strcmp(nm, "padding")) p->padding = v;
    else if (!std::strcmp(nm, "dilation")) p->dilation = v;
    else if (!std::strcmp(nm, "kernel")) p->kernel = v;
    else if (!std::strcmp(nm, "deformable_groups")) p->deformable_groups = v;
  }
  return p;
}

dcnv2_plugin* dcnv2_plugin_clone(const dcnv2_plugin* p) {
  if (!p) return nullptr;
  return new (std::nothrow) dcnv2_plugin(*p);
}

void dcnv2_plugin_destroy(dcnv2_plugin* p) { delete p; }

int32_t dcnv2_plugin_serialize(const dcnv2_plugin* p, const char** names, int32_t values[5]) {
  if (!p || !values) return 0;
  values[0] = p->stride;
  values[1] = p->padding;
  values[2] = p->dilation;
  values[3] = p->kernel;
  values[4] = p->deformable_groups;
  if (names)
    for (int i = 0; i < 5; ++i) names[i] = kFieldNames[i];
  return 5;
}

int32_t dcnv2_plugin_nb_outputs(const dcnv2_plugin*) { return 1; }

int32_t dcnv2_plugin_output_dtype(const dcnv2_plugin*, int32_t x_type) {
  return x_type == DCNV2_INT8 ? DCNV2_FLOAT : x_type;
}

dcnv2_status dcnv2_plugin_output_shape(const dcnv2_plugin* p, const int64_t x_dims[4],
                                       const int64_t w_dims[4], int64_t out_dims[4]) {
  if (!p || !x_dims || !w_dims || !out_dims) return DCNV2_ERR_INVALID_ARG;
  if (p->stride < 1) return DCNV2_ERR_INVALID_ARG;
  const int64_t c = 2 * int64_t(p->padding) - int64_t(p->dilation) * (p->kernel - 1) - 1;
  auto out_dim = [&](int64_t in) -> int64_t {
    const int64_t t = in + c;
    // kFLOOR_DIV semantics (src/dcn_plugin.cpp:80): floor for negative numerators too.
    const int64_t q = t >= 0 ? t / p->stride : -((-t + p->stride - 1) / p->stride);
    return q + 1;
  };
  out_dims[0] = x_dims[0];
  out_dims[1] = w_dims[0];
  out_dims[2] = out_dim(x_dims[2]);
  out_dims[3] = out_dim(x_dims[3]);
  return DCNV2_OK;
}

int32_t dcnv2_plugin_supports_format(const dcnv2_plugin* p, int32_t pos,
                                     const dcnv2_tensor_desc* in_out, int32_t nb_inputs,
                                     int32_t nb_outputs) {
  if (!p || !in_out || pos < 0 || pos >= nb_inputs + nb_outputs) return 0;
  if (in_out[pos].format != DCNV2_FORMAT_LINEAR) return 0;
  const int32_t t = in_out[pos].type;
  if (pos == 0) return type_ok(t) ? 1 : 0;
  const int32_t t0 = in_out[0].type;
  if (t0 == DCNV2_INT8) return (pos == 3) ? (t == DCNV2_INT8) : (t == DCNV2_FLOAT);
  return t == t0 ? 1 : 0;
}

static bool desc_from_tensors(const dcnv2_plugin* p, const dcnv2_tensor_desc* in,
                              const dcnv2_tensor_desc* w, dcnv2_desc* d) {
  if (!p || !in || !w || in->nb_dims != 4 || w->nb_dims < 1) return false;
  d->n = to_i32(in->d[0]);
  d->c = to_i32(in->d[1]);
  d->h = to_i32(in->d[2]);
  d->w = to_i32(in->d[3]);
  d->out_c = to_i32(w->d[0]);
  d->kernel = p->kernel;
  d->stride = p->stride;
  d->padding = p->padding;
  d->dilation = p->dilation;
  d->deformable_groups = p->deformable_groups;
  d->dtype = in->type;
  d->math = DCNV2_MATH_DEFAULT;
  return true;
}

size_t dcnv2_plugin_workspace_size(const dcnv2_plugin* p, const dcnv2_tensor_desc* inputs,
                                   int32_t nb_inputs, const dcnv2_tensor_desc* outputs,
                                   int32_t nb_outputs) {
  if (!p || !inputs || nb_inputs < 5 || !outputs || nb_outputs < 1) return 0;
  dcnv2_desc d;
  if (!desc_from_tensors(p, &inputs[0], &inputs[3], &d)) return 0;
  return dcnv2_workspace_size(&d);
}

int32_t dcnv2_plugin_enqueue(const dcnv2_plugin* p, const dcnv2_tensor_desc* in_desc,
                             const dcnv2_tensor_desc* out_desc, const void* const* inputs,
                             void* const* outputs, void* workspace, size_t workspace_bytes,
                             dcnv2_stream_t stream) {
  if (!p || !in_desc || !out_desc || !inputs || !outputs) return DCNV2_ERR_INVALID_ARG;
  dcnv2_desc d;
  if (!desc_from_tensors(p, &in_desc[0], &in_desc[3], &d)) return DCNV2_ERR_INVALID_ARG;
  // The output shape TensorRT bound must be the one getOutputShapes derives.
  int64_t expect[4];
  if (dcnv2_output_shape(&d, expect) != DCNV2_OK) return DCNV2_ERR_INVALID_ARG;
  if (out_desc[0].nb_dims != 4) return DCNV2_ERR_INVALID_ARG;
  for (int i = 0; i < 4; ++i)
    if (out_desc[0].d[i] != expect[i]) return DCNV2_ERR_INVALID_ARG;
  // Precision combination must be one that supportsFormatCombination accepts.
  dcnv2_tensor_desc all[6];
  for (int i = 0; i < 5; ++i) all[i] = in_desc[i];
  all[5] = out_desc[0];
  for (int pos = 0; pos < 6; ++pos)
    if (!dcnv2_plugin_supports_format(p, pos, all, 5, 1)) return DCNV2_ERR_UNSUPPORTED;
  const float xs = in_desc[0].scale, ws = in_desc[3].scale;
  return dcnv2_forward(&d, inputs[0], inputs[1], inputs[2], inputs[3], inputs[4], outputs[0],
                       workspace, workspace_bytes, xs, ws, stream);
}

}  // extern "C"
