// moe_prefill.cu — placeholder while the grouped tcgen05 path is written.
#include "common.cuh"
extern "C" size_t iq36_moe_prefill_workspace_bytes(int32_t, int32_t, int32_t, int32_t, int32_t) { return 256; }
extern "C" int iq36_moe_prefill(const void*, int32_t, const int32_t*, const float*, int32_t,
                                const iq36_expert_bank*, void*, int32_t, void*, size_t, iq36_stream_t) {
  return IQ36_ERR_SHAPE;
}
