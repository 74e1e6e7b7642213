// K2: attention backward (placeholder until the tcgen05 kernel lands).
#include "kf_host.h"

extern "C" size_t kf_attn_bwd_workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t D) {
  return (size_t)(B * Hq * Sq) * (size_t)(D + 1) * sizeof(float) + 256;
}

extern "C" int kf_attn_bwd(const kf_tensor4*, const kf_tensor4*, const kf_tensor4*,
                           const kf_tensor4*, const float*, const kf_tensor4*,
                           const kf_tensor4*, const kf_tensor4*, const kf_tensor4*, int, float,
                           int, void*, size_t, int32_t*, void*) {
  return kf::set_error(KF_ERR_UNSUPPORTED, "kf_attn_bwd: not built yet");
}
