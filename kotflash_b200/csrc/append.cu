// K4: KV-cache append.  One launch copies new_k -> k_cache and new_v -> v_cache
// at sequence offset `start` (replaces append_kv_kernel + append_kv_cuda,
// kotflash/csrc/kv_append_cuda.cu:12-96).  Each thread moves one 16-byte
// vector of K and one of V (eight 16-bit elements), so a warp writes 512
// contiguous bytes of a cache row; views whose rows are not 16-byte aligned
// take the element-wise variant.  Pure data movement: bit-exact.
#include "kf_host.h"
#include "kf_sm100.cuh"

namespace {

struct AppendArgs {
  const uint16_t* src_k;
  const uint16_t* src_v;
  uint16_t* dst_k;
  uint16_t* dst_v;
  int64_t H, S, D, start;
  int64_t sk[4], sv[4], dk[4], dv[4];
};

template <int VEC>
__global__ void __launch_bounds__(256) append_kernel(AppendArgs a, int64_t total_vecs) {
  const int64_t dvecs = a.D / VEC;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total_vecs;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t dv_i = i % dvecs;
    const int64_t row = i / dvecs;
    const int64_t t = row % a.S;
    const int64_t bh = row / a.S;
    const int64_t h = bh % a.H;
    const int64_t b = bh / a.H;
    const int64_t d = dv_i * VEC;
    const int64_t ok = b * a.sk[0] + h * a.sk[1] + t * a.sk[2] + d * a.sk[3];
    const int64_t ov = b * a.sv[0] + h * a.sv[1] + t * a.sv[2] + d * a.sv[3];
    const int64_t odk = b * a.dk[0] + h * a.dk[1] + (a.start + t) * a.dk[2] + d * a.dk[3];
    const int64_t odv = b * a.dv[0] + h * a.dv[1] + (a.start + t) * a.dv[2] + d * a.dv[3];
    if constexpr (VEC == 8) {
      const uint4 kv = __ldg(reinterpret_cast<const uint4*>(a.src_k + ok));
      const uint4 vv = __ldg(reinterpret_cast<const uint4*>(a.src_v + ov));
      *reinterpret_cast<uint4*>(a.dst_k + odk) = kv;
      *reinterpret_cast<uint4*>(a.dst_v + odv) = vv;
    } else {
      a.dst_k[odk] = a.src_k[ok];
      a.dst_v[odv] = a.src_v[ov];
    }
  }
}

bool vec_ok(const kf_tensor4* t) {
  if (!kf::aligned16(t->ptr) || t->stride[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (t->size[i] > 1 && (t->stride[i] % 8) != 0) return false;
  return true;
}

}  // namespace

extern "C" int kf_append(const kf_tensor4* k_cache, const kf_tensor4* v_cache,
                         const kf_tensor4* new_k, const kf_tensor4* new_v, int64_t start,
                         int dtype, void* stream) {
  using kf::set_error;
  if (!k_cache || !v_cache || !new_k || !new_v)
    return set_error(KF_ERR_INVALID, "kf_append: null tensor descriptor");
  if (dtype != KF_F16 && dtype != KF_BF16)
    return set_error(KF_ERR_INVALID, "kf_append: dtype must be fp16 or bf16");
  for (int i = 0; i < 4; ++i) {
    if (k_cache->size[i] != v_cache->size[i])
      return set_error(KF_ERR_INVALID, "kf_append: K/V cache shapes must match");
    if (new_k->size[i] != new_v->size[i])
      return set_error(KF_ERR_INVALID, "kf_append: new K/V shapes must match");
  }
  const int64_t B = new_k->size[0], H = new_k->size[1], S = new_k->size[2], D = new_k->size[3];
  if (B != k_cache->size[0] || H != k_cache->size[1] || D != k_cache->size[3])
    return set_error(KF_ERR_INVALID, "kf_append: new K/V batch, heads and head_dim must match the cache");
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0)
    return set_error(KF_ERR_INVALID, "kf_append: new K/V dimensions must be non-empty");
  if (start < 0 || start + S > k_cache->size[2])
    return set_error(KF_ERR_INVALID, "kf_append: append range exceeds cache capacity");
  if (!k_cache->ptr || !v_cache->ptr || !new_k->ptr || !new_v->ptr)
    return set_error(KF_ERR_INVALID, "kf_append: null data pointer");
  kf::DeviceGuard guard(k_cache->ptr);
  if (guard.status()) return guard.status();

  AppendArgs a;
  a.src_k = static_cast<const uint16_t*>(new_k->ptr);
  a.src_v = static_cast<const uint16_t*>(new_v->ptr);
  a.dst_k = static_cast<uint16_t*>(k_cache->ptr);
  a.dst_v = static_cast<uint16_t*>(v_cache->ptr);
  a.H = H;
  a.S = S;
  a.D = D;
  a.start = start;
  for (int i = 0; i < 4; ++i) {
    a.sk[i] = new_k->stride[i];
    a.sv[i] = new_v->stride[i];
    a.dk[i] = k_cache->stride[i];
    a.dv[i] = v_cache->stride[i];
  }
  const bool vec = (D % 8 == 0) && vec_ok(k_cache) && vec_ok(v_cache) && vec_ok(new_k) &&
                   vec_ok(new_v);
  const int64_t total = B * H * S * (vec ? D / 8 : D);
  const int threads = 256;
  const int64_t max_blocks = (int64_t)kf::sm_count_current_device() * 16;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > max_blocks) blocks = max_blocks;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (vec)
    append_kernel<8><<<(unsigned)blocks, threads, 0, st>>>(a, total);
  else
    append_kernel<1><<<(unsigned)blocks, threads, 0, st>>>(a, total);
  return kf::check_launch("kf_append");
}
