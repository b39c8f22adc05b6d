// placeholder, replaced by the tcgen05 implementation
#include "common.cuh"
using namespace crb;
extern "C" int cr_filtered_topk(const uint16_t*, const float*, uint64_t, uint32_t, const uint16_t*,
                                uint32_t, const cr_gpu_roaring*, uint64_t, uint32_t, int, float*,
                                int64_t*, cr_stream_t)
{
  set_last_error("cr_filtered_topk: not built yet");
  return CR_ERR_UNSUPPORTED;
}
extern "C" int cr_row_norms(const uint16_t*, uint64_t, uint32_t, float*, cr_stream_t)
{
  set_last_error("cr_row_norms: not built yet");
  return CR_ERR_UNSUPPORTED;
}
extern "C" int cr_topk_merge(const float*, const int64_t*, uint32_t, uint32_t, uint32_t, int,
                             float*, int64_t*, cr_stream_t)
{
  set_last_error("cr_topk_merge: not built yet");
  return CR_ERR_UNSUPPORTED;
}
