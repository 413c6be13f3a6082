// KV append: scatter of the step's new K/V rows into the block pools.
//
// Same effect as PagedKVCache.append (jyotilakra92/nifre
// src/inference/paged_kv_cache.py:107-121): for every new token,
// k[layer][block, offset] = key[token] (cast to the cache dtype), through the
// destination rows computed once per step by nf_pack_step instead of a Python
// resolve() per token.  HBM-bound: every thread moves 16-byte vectors; one
// pool row (num_kv_heads * head_dim elements) is contiguous in both tensors.
#include "nf_common.cuh"
#include "nf_internal.h"

namespace nf {

struct AppendParams {
  char* kp;
  char* vp;
  long long pool_rows;
  const char* kn;
  const char* vn;
  long long ks, vs;  // source row strides (elements)
  const int* slot_mapping;
  const int* src_rows;
  int n_tokens;
  int row_elems;
  const int* seqs;
  int n_seqs;
  long long* pos_out;
  int* status;
};

template <typename T> struct Vec8;  // 8 elements loaded/stored as wide vectors
template <> struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&x)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&x)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
  }
};
template <typename H> struct Vec8Half {
  static __device__ __forceinline__ void load(const H* p, float (&x)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const H* h = reinterpret_cast<const H*>(&a);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = Elem<H>::to_f(h[i]);
  }
  static __device__ __forceinline__ void store(H* p, const float (&x)[8]) {
    uint4 a;
    H* h = reinterpret_cast<H*>(&a);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = Elem<H>::from_f(x[i]);
    *reinterpret_cast<uint4*>(p) = a;
  }
};
template <> struct Vec8<__half> : Vec8Half<__half> {};
template <> struct Vec8<__nv_bfloat16> : Vec8Half<__nv_bfloat16> {};

// Same-type rows: raw 16-byte copies (bit exact by construction).
template <typename T>
__global__ void append_copy_kernel(const AppendParams p) {
  pdl_launch_dependents();
  pdl_wait();  // the rows may come from the launch before this one
  constexpr int V = 16 / sizeof(T);
  const int chunks = p.row_elems / V;
  const long long total = (long long)p.n_tokens * 2 * chunks;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(idx % chunks);
    const long long r = idx / chunks;
    const int t = (int)(r >> 1), kv = (int)(r & 1);
    const int slot = p.slot_mapping[t];
    if (slot < 0 || slot >= p.pool_rows) {
      atomicOr(p.status, NF_STATUS_BAD_SLOT);
      continue;
    }
    const long long srow = p.src_rows[t];
    const T* src = reinterpret_cast<const T*>(kv ? p.vn : p.kn) + srow * (kv ? p.vs : p.ks) + c * V;
    T* dst = reinterpret_cast<T*>(kv ? p.vp : p.kp) + (long long)slot * p.row_elems + c * V;
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
  }
  if (p.pos_out && blockIdx.x == 0) {
    for (int s = threadIdx.x; s < p.n_seqs; s += blockDim.x)
      p.pos_out[p.seqs[4 * s]] = (long long)p.seqs[4 * s + 3] + p.seqs[4 * s + 2];
  }
}

// Converting rows (e.g. float32 projections into a bfloat16 pool):
// round-to-nearest-even per element like torch's copy_.
template <typename Ts, typename Td>
__global__ void append_convert_kernel(const AppendParams p) {
  pdl_launch_dependents();
  pdl_wait();  // the rows may come from the launch before this one
  const int chunks = p.row_elems / 8;
  const long long total = (long long)p.n_tokens * 2 * chunks;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(idx % chunks);
    const long long r = idx / chunks;
    const int t = (int)(r >> 1), kv = (int)(r & 1);
    const int slot = p.slot_mapping[t];
    if (slot < 0 || slot >= p.pool_rows) {
      atomicOr(p.status, NF_STATUS_BAD_SLOT);
      continue;
    }
    const long long srow = p.src_rows[t];
    const Ts* src = reinterpret_cast<const Ts*>(kv ? p.vn : p.kn) + srow * (kv ? p.vs : p.ks) + c * 8;
    Td* dst = reinterpret_cast<Td*>(kv ? p.vp : p.kp) + (long long)slot * p.row_elems + c * 8;
    float x[8];
    Vec8<Ts>::load(src, x);
    Vec8<Td>::store(dst, x);
  }
  if (p.pos_out && blockIdx.x == 0) {
    for (int s = threadIdx.x; s < p.n_seqs; s += blockDim.x)
      p.pos_out[p.seqs[4 * s]] = (long long)p.seqs[4 * s + 3] + p.seqs[4 * s + 2];
  }
}

// Rows whose length or alignment does not allow vectors: one element per thread.
template <typename Ts, typename Td>
__global__ void append_scalar_kernel(const AppendParams p) {
  pdl_launch_dependents();
  pdl_wait();  // the rows may come from the launch before this one
  const long long total = (long long)p.n_tokens * 2 * p.row_elems;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int e = (int)(idx % p.row_elems);
    const long long r = idx / p.row_elems;
    const int t = (int)(r >> 1), kv = (int)(r & 1);
    const int slot = p.slot_mapping[t];
    if (slot < 0 || slot >= p.pool_rows) {
      atomicOr(p.status, NF_STATUS_BAD_SLOT);
      continue;
    }
    const long long srow = p.src_rows[t];
    const Ts* src = reinterpret_cast<const Ts*>(kv ? p.vn : p.kn) + srow * (kv ? p.vs : p.ks);
    Td* dst = reinterpret_cast<Td*>(kv ? p.vp : p.kp) + (long long)slot * p.row_elems;
    dst[e] = Elem<Td>::from_f(Elem<Ts>::to_f(src[e]));
  }
  if (p.pos_out && blockIdx.x == 0) {
    for (int s = threadIdx.x; s < p.n_seqs; s += blockDim.x)
      p.pos_out[p.seqs[4 * s]] = (long long)p.seqs[4 * s + 3] + p.seqs[4 * s + 2];
  }
}

// The append kernels launch with programmatic stream serialization: a grid
// may start while the launch before it on the stream (the previous layer's
// attention) finishes, and waits for it (griddepcontrol.wait) before reading
// anything, so its launch and start-up overlap that kernel's tail.  Plain
// stream order where the launch refuses the attribute.
template <typename K>
static void launch_pdl(K kern, long long blocks, int threads, cudaStream_t st, const AppendParams& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) {
    (void)cudaGetLastError();
    kern<<<(unsigned)blocks, threads, 0, st>>>(p);
  }
}

template <typename Ts, typename Td>
static void launch_append(const AppendParams& p, bool vec_ok, cudaStream_t st) {
  const int threads = 256;
  const long long work = (long long)p.n_tokens * 2 * (vec_ok ? p.row_elems / 8 : p.row_elems);
  long long blocks = (work + threads - 1) / threads;
  const long long cap = (long long)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (!vec_ok) {
    launch_pdl(append_scalar_kernel<Ts, Td>, blocks, threads, st, p);
  } else if (sizeof(Ts) == sizeof(Td) && std::is_same<Ts, Td>::value) {
    const long long vwork = (long long)p.n_tokens * 2 * (p.row_elems * sizeof(Td) / 16);
    long long vb = (vwork + threads - 1) / threads;
    if (vb > cap) vb = cap;
    if (vb < 1) vb = 1;
    launch_pdl(append_copy_kernel<Td>, vb, threads, st, p);
  } else {
    launch_pdl(append_convert_kernel<Ts, Td>, blocks, threads, st, p);
  }
}

template <typename Ts>
static int dispatch_dst(int dst, const AppendParams& p, bool vec_ok, cudaStream_t st) {
  switch (dst) {
    case NF_F32: launch_append<Ts, float>(p, vec_ok, st); break;
    case NF_F16: launch_append<Ts, __half>(p, vec_ok, st); break;
    case NF_BF16: launch_append<Ts, __nv_bfloat16>(p, vec_ok, st); break;
    default: return fail(NF_EINVAL, "nf_kv_append: bad pool dtype %d", dst);
  }
  return check_launch("nf_kv_append");
}

}  // namespace nf

extern "C" int nf_kv_append(void* k_pool, void* v_pool, int32_t pool_dtype, int64_t pool_rows,
                            const void* k_new, const void* v_new, int32_t src_dtype,
                            int64_t k_src_row_stride, int64_t v_src_row_stride,
                            const int32_t* slot_mapping, const int32_t* src_rows, int32_t n_tokens,
                            int32_t num_kv_heads, int32_t head_dim, const int32_t* seqs, int32_t n_seqs,
                            int64_t* pos_out, int32_t* status, void* stream) {
  using namespace nf;
  if (n_tokens <= 0) return fail(NF_EINVAL, "nf_kv_append: n_tokens must be positive");
  if (!k_pool || !v_pool || !k_new || !v_new || !slot_mapping || !src_rows || !status)
    return fail(NF_EINVAL, "nf_kv_append: null pointer argument");
  if (pos_out && (!seqs || n_seqs <= 0)) return fail(NF_EINVAL, "nf_kv_append: pos_out needs seqs");
  const size_t es = dtype_size(src_dtype), ed = dtype_size(pool_dtype);
  if (!es || !ed) return fail(NF_EINVAL, "nf_kv_append: bad dtype (src %d, pool %d)", src_dtype, pool_dtype);
  if (num_kv_heads <= 0 || head_dim <= 0 || pool_rows <= 0) return fail(NF_EINVAL, "nf_kv_append: sizes must be positive");
  AppendParams p;
  p.kp = static_cast<char*>(k_pool);
  p.vp = static_cast<char*>(v_pool);
  p.pool_rows = pool_rows;
  p.kn = static_cast<const char*>(k_new);
  p.vn = static_cast<const char*>(v_new);
  p.ks = k_src_row_stride;
  p.vs = v_src_row_stride;
  p.slot_mapping = slot_mapping;
  p.src_rows = src_rows;
  p.n_tokens = n_tokens;
  p.row_elems = num_kv_heads * head_dim;
  p.seqs = seqs;
  p.n_seqs = pos_out ? n_seqs : 0;
  p.pos_out = reinterpret_cast<long long*>(pos_out);
  p.status = status;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  const bool vec_ok = (p.row_elems % 8 == 0) && al16(k_pool) && al16(v_pool) && al16(k_new) && al16(v_new) &&
                      ((k_src_row_stride * (long long)es) % 16 == 0) && ((v_src_row_stride * (long long)es) % 16 == 0) &&
                      ((p.row_elems * ed) % 16 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (src_dtype) {
    case NF_F32: return dispatch_dst<float>(pool_dtype, p, vec_ok, st);
    case NF_F16: return dispatch_dst<__half>(pool_dtype, p, vec_ok, st);
    case NF_BF16: return dispatch_dst<__nv_bfloat16>(pool_dtype, p, vec_ok, st);
  }
  return fail(NF_EINVAL, "nf_kv_append: bad src dtype %d", src_dtype);
}

extern "C" int nf_kv_append_args(const NfAppendArgs* a, void* stream) {
  if (!a) return nf::fail(NF_EINVAL, "nf_kv_append_args: null argument struct");
  return nf_kv_append(a->k_pool, a->v_pool, a->pool_dtype, a->pool_rows, a->k_new, a->v_new, a->src_dtype,
                      a->k_src_row_stride, a->v_src_row_stride, a->slot_mapping, a->src_rows, a->n_tokens,
                      a->num_kv_heads, a->head_dim, a->seqs, a->n_seqs, a->pos_out, a->status, stream);
}
