// hd_decoder.cu -- placeholder.
#include "hd_internal.cuh"
extern "C" int hd_decoder_create(hd_ctx *ctx, const hd_decoder_config *, const hd_layer_weights *, const float *,
                                 const hd_weight *, hd_decoder **out) {
    if (out) *out = nullptr;
    return hd_fail(ctx, HD_E_UNSUPPORTED, "decoder not built yet");
}
extern "C" int hd_decoder_free(hd_decoder *) { return HD_OK; }
extern "C" int hd_decoder_generate(hd_decoder *, const int32_t *, int, int, int, int, int32_t *, float *, float *) {
    return HD_E_UNSUPPORTED;
}
