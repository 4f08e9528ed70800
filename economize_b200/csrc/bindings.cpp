// PyTorch bindings of the economize_b200 sm_100a kernels (module economize_b200._C).
//
// Each op checks devices, dtypes and shapes, builds the TMA descriptors it needs (cached per pointer and shape),
// allocates outputs and workspaces through PyTorch's caching allocator (so CUDA-graph capture works) and launches
// on the current stream. A launcher that refuses a shape raises a Python error; nothing falls back to PyTorch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <list>
#include <string>
#include <mutex>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "launchers.h"

namespace {

using at::Tensor;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bfloat16")
// every tensor a kernel dereferences must live on the launching tensor's CUDA device (a host pointer faults)
#define CHECK_ON(x, ref)                                                                                         \
  TORCH_CHECK((x).is_cuda() && (x).get_device() == (ref).get_device(), #x " must be on the device of " #ref)
#define CHECK_I32(x) TORCH_CHECK((x).scalar_type() == at::kInt, #x " must be int32")
#define CHECK_I64(x) TORCH_CHECK((x).scalar_type() == at::kLong, #x " must be int64")

int num_sms(int device) {
  static std::vector<int> cache(64, 0);
  if (cache[device] == 0) {
    cudaDeviceGetAttribute(&cache[device], cudaDevAttrMultiProcessorCount, device);
  }
  return cache[device];
}

// Per-device status word that kernels set when a bounded wait gives up.
unsigned* status_word(const at::Device& device) {
  static std::mutex mu;
  static std::unordered_map<int, Tensor> words;
  std::lock_guard<std::mutex> lock(mu);
  auto it = words.find(device.index());
  if (it == words.end()) {
    it = words.emplace(device.index(), at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(device))).first;
  }
  return reinterpret_cast<unsigned*>(it->second.data_ptr<int>());
}

// Split-K tile counters (zeroed once, reset by the kernels) private to each (device, stream).
int* split_counters(const at::Device& device, cudaStream_t stream) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, Tensor> bufs;
  std::lock_guard<std::mutex> lock(mu);
  const uint64_t key = (static_cast<uint64_t>(device.index()) << 56) ^ reinterpret_cast<uint64_t>(stream);
  auto it = bufs.find(key);
  if (it == bufs.end()) {
    it = bufs.emplace(key, at::zeros({8192}, at::TensorOptions().dtype(at::kInt).device(device))).first;
  }
  return it->second.data_ptr<int>();
}

// Arrival counters of kernels whose last CTA finishes a reduction (zeroed once; every such kernel leaves them
// zero), one buffer per device, stream and user: 0 = split top-k (per row).
constexpr int kCounterInts[1] = {1024};

int* arrival_counters(const at::Device& device, cudaStream_t stream, int which) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, Tensor> bufs;
  std::lock_guard<std::mutex> lock(mu);
  const uint64_t key = ((static_cast<uint64_t>(device.index()) << 56) ^ reinterpret_cast<uint64_t>(stream)) * 4 +
                       static_cast<uint64_t>(which);
  auto it = bufs.find(key);
  if (it == bufs.end()) {
    it = bufs.emplace(key, at::zeros({kCounterInts[which]}, at::TensorOptions().dtype(at::kInt).device(device)))
             .first;
  }
  return it->second.data_ptr<int>();
}

// LRU cache of tensor maps keyed by (base, element size, shape, stride, box, swizzle).
struct MapKey {
  uintptr_t base;
  uint64_t rows, cols, stride;
  uint32_t box_cols, box_rows;
  int elem, swizzle;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && stride == o.stride && box_cols == o.box_cols &&
           box_rows == o.box_rows && elem == o.elem && swizzle == o.swizzle;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.base) ^ (k.rows * 1315423911u) ^ (k.cols << 7) ^ (k.stride << 17) ^
           (static_cast<uint64_t>(k.box_rows) << 3) ^ (static_cast<uint64_t>(k.box_cols) << 40) ^ (k.elem << 29) ^
           (static_cast<uint64_t>(k.swizzle) << 50);
  }
};

// Tensor map of a row-major [rows, cols] matrix of `elem`-byte elements (row stride in bytes).
const CUtensorMap* tensor_map_ex(const void* base, int elem, uint64_t rows, uint64_t cols, uint64_t stride_bytes,
                                 uint32_t box_cols, uint32_t box_rows, int swizzle) {
  static std::mutex mu;
  static std::list<std::pair<MapKey, CUtensorMap>> lru;
  static std::unordered_map<MapKey, std::list<std::pair<MapKey, CUtensorMap>>::iterator, MapKeyHash> index;
  constexpr size_t kCap = 4096;
  std::lock_guard<std::mutex> lock(mu);
  MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, stride_bytes, box_cols, box_rows, elem, swizzle};
  auto it = index.find(key);
  if (it != index.end()) {
    lru.splice(lru.begin(), lru, it->second);
    return &it->second->second;
  }
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  const int rc = ecz::make_tmap_2d(&map, elem, base, rows, cols, stride_bytes, box_cols, box_rows, swizzle);
  TORCH_CHECK(rc == 0, "cuTensorMapEncodeTiled failed (code ", rc, ") for rows=", rows, " cols=", cols);
  lru.emplace_front(key, map);
  index[key] = lru.begin();
  if (lru.size() > kCap) {
    index.erase(lru.back().first);
    lru.pop_back();
  }
  return &lru.front().second;
}

// bf16 [rows, cols] (row stride in elements) with a {64, box} box and the 128-byte swizzle: the GEMM/attention
// operand layout.
const CUtensorMap* tensor_map(const void* base, uint64_t rows, uint64_t cols, uint64_t stride, uint32_t box) {
  return tensor_map_ex(base, 2, rows, cols, stride * 2, 64, box, 128);
}

// A split-K partials input is an fp32 tensor with one extra leading dimension [splits, ...] (see linear_parts);
// returns (splits, the bf16 shape it stands for).
std::pair<int, std::vector<int64_t>> parts_of(const Tensor& x) {
  if (x.scalar_type() == at::kBFloat16) return {0, x.sizes().vec()};
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.dim() >= 2 && x.is_contiguous() && x.size(0) <= 8,
              "expected a bf16 tensor or contiguous fp32 split-K partials [splits <= 8, ...]");
  return {static_cast<int>(x.size(0)), std::vector<int64_t>(x.sizes().begin() + 1, x.sizes().end())};
}

std::tuple<Tensor, Tensor> rmsnorm(Tensor x, Tensor w, double eps, c10::optional<Tensor> resid) {
  CHECK_CUDA(x);
  CHECK_BF16(w);
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  const auto [splits, shape] = parts_of(x);
  const int hidden = static_cast<int>(shape.back());
  int64_t numel = 1;
  for (auto d : shape) numel *= d;
  const int rows = static_cast<int>(numel / hidden);
  Tensor r;
  if (resid.has_value()) {
    r = resid->contiguous();
    CHECK_BF16(r);
    TORCH_CHECK(r.numel() == numel, "residual shape mismatch");
  }
  const auto opts = x.options().dtype(at::kBFloat16);
  auto out = at::empty(shape, opts);
  auto resid_out = at::empty(shape, opts);
  const int rc = ecz::launch_rmsnorm(splits ? nullptr : x.data_ptr(), resid.has_value() ? r.data_ptr() : nullptr,
                                     w.data_ptr(), out.data_ptr(), resid_out.data_ptr(), rows, hidden,
                                     static_cast<float>(eps), at::cuda::getCurrentCUDAStream(),
                                     splits ? x.data_ptr<float>() : nullptr, splits);
  TORCH_CHECK(rc == 0, "rmsnorm: unsupported hidden size ", hidden);
  return {out, resid_out};
}

// fp8 scales: per-KV-head fp32 [Hkv] (K = k_scale * K8, V = v_scale * V8) when the caches hold e4m3 codes.
bool fp8_cache(const Tensor& k_cache, const c10::optional<Tensor>& k_scale, const c10::optional<Tensor>& v_scale,
               int64_t Hkv) {
  if (k_cache.scalar_type() == at::kBFloat16) return false;
  TORCH_CHECK(k_cache.scalar_type() == at::kFloat8_e4m3fn, "caches must be bf16 or float8_e4m3fn");
  TORCH_CHECK(k_scale.has_value() && v_scale.has_value(), "fp8 caches need k_scale and v_scale");
  for (const Tensor* t : {&*k_scale, &*v_scale}) {
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == Hkv,
                "fp8 scales must be contiguous fp32 [Hkv]");
  }
  return true;
}

// One layer's K or V cache argument: a contiguous [B, Hkv, S, D] tensor, or, with a page table [B, C] (int32), a view
// [P, Hkv, 128, D] of a page pool whose pages start stride(0) elements apart (dims 1-3 packed). Gives the logical
// capacity S, the kernels' page description and the rows a 2-D TMA map over the view may address.
struct CacheArg {
  int S = 0;
  uint64_t rows = 0;
  ecz::KVPages pages;
};

CacheArg cache_arg(const Tensor& cache, const c10::optional<Tensor>& table, int64_t B, const char* what) {
  TORCH_CHECK(cache.dim() == 4, what, ": caches must be 4-D ([B, Hkv, S, D], or page-pool views [P, Hkv, 128, D])");
  const int64_t Hkv = cache.size(1), D = cache.size(3);
  CacheArg a;
  if (!table.has_value()) {
    TORCH_CHECK(cache.is_contiguous(), what, ": caches must be contiguous");
    a.S = static_cast<int>(cache.size(2));
    a.rows = static_cast<uint64_t>(cache.size(0)) * Hkv * a.S;
    return a;
  }
  CHECK_I32(*table);
  CHECK_ON(*table, cache);
  TORCH_CHECK(table->dim() == 2 && table->size(0) == B && table->is_contiguous(), what,
              ": page tables must be contiguous int32 [B, chunks]");
  TORCH_CHECK(cache.size(2) == 128 && cache.stride(3) == 1 && cache.stride(2) == D && cache.stride(1) == 128 * D &&
                  cache.stride(0) % (128 * D) == 0 && cache.stride(0) >= Hkv * 128 * D,
              what, ": a paged cache must be a view [P, Hkv, 128, D] of whole pages");
  a.S = static_cast<int>(table->size(1) * 128);
  a.pages.table = table->data_ptr<int>();
  a.pages.max_chunks = static_cast<int>(table->size(1));
  a.pages.page_rows = static_cast<int>(cache.stride(0) / D);
  a.rows = static_cast<uint64_t>(cache.size(0) - 1) * a.pages.page_rows + static_cast<uint64_t>(Hkv) * 128;
  return a;
}

// A whole cache (every layer): contiguous [L, 2, B, Hkv, S, D], or a page pool [P, 2, Hkv, 128, D] with page tables
// [L, B, C] (int32).
struct WholeCache {
  int L = 0, B = 0, Hkv = 0, S = 0, D = 0;
  ecz::KVLayout layout;
};

WholeCache whole_cache(const Tensor& cache, const c10::optional<Tensor>& tables, const char* what) {
  TORCH_CHECK(cache.is_contiguous(), what, ": the cache must be contiguous");
  WholeCache w;
  if (!tables.has_value()) {
    TORCH_CHECK(cache.dim() == 6, what, ": the cache must be [L, 2, B, Hkv, S, D]");
    w.L = static_cast<int>(cache.size(0));
    w.B = static_cast<int>(cache.size(2));
    w.Hkv = static_cast<int>(cache.size(3));
    w.S = static_cast<int>(cache.size(4));
    w.D = static_cast<int>(cache.size(5));
    w.layout.v_rows = static_cast<long>(w.B) * w.Hkv * w.S;
    w.layout.layer_rows = 2 * w.layout.v_rows;
    return w;
  }
  CHECK_I32(*tables);
  CHECK_ON(*tables, cache);
  TORCH_CHECK(cache.dim() == 5 && cache.size(1) == 2 && cache.size(3) == 128, what,
              ": a paged cache must be a pool [P, 2, Hkv, 128, D]");
  TORCH_CHECK(tables->dim() == 3 && tables->is_contiguous(), what, ": page tables must be int32 [L, B, chunks]");
  w.L = static_cast<int>(tables->size(0));
  w.B = static_cast<int>(tables->size(1));
  w.Hkv = static_cast<int>(cache.size(2));
  w.S = static_cast<int>(tables->size(2) * 128);
  w.D = static_cast<int>(cache.size(4));
  w.layout.pages.table = tables->data_ptr<int>();
  w.layout.pages.max_chunks = static_cast<int>(tables->size(2));
  w.layout.pages.page_rows = 2 * w.Hkv * 128;
  w.layout.table_stride = static_cast<long>(w.B) * tables->size(2);
  w.layout.layer_rows = 0;
  w.layout.v_rows = static_cast<long>(w.Hkv) * 128;
  return w;
}

Tensor rope_store(Tensor qkv, Tensor positions, Tensor cos, Tensor sin, int64_t H, int64_t Hkv, int64_t D,
                  Tensor k_cache, Tensor v_cache, Tensor kv_len, Tensor n_new, c10::optional<Tensor> q_norm,
                  c10::optional<Tensor> k_norm, double eps, int64_t q_offset, c10::optional<Tensor> k_scale,
                  c10::optional<Tensor> v_scale, c10::optional<Tensor> pages) {
  CHECK_CUDA(qkv);
  TORCH_CHECK(D == 64 || D == 128 || D == 256, "rope_store: head_dim must be 64, 128 or 256, got ", D);
  const auto [qkv_splits, qkv_shape] = parts_of(qkv);
  const bool fp8 = fp8_cache(k_cache, k_scale, v_scale, Hkv);
  TORCH_CHECK(v_cache.scalar_type() == k_cache.scalar_type(), "K and V caches must share a dtype");
  CHECK_I32(positions);
  CHECK_I32(kv_len);
  CHECK_I32(n_new);
  CHECK_ON(positions, qkv);
  CHECK_ON(kv_len, qkv);
  CHECK_ON(n_new, qkv);
  CHECK_ON(cos, qkv);
  CHECK_ON(sin, qkv);
  CHECK_ON(k_cache, qkv);
  CHECK_ON(v_cache, qkv);
  TORCH_CHECK(cos.scalar_type() == at::kFloat && sin.scalar_type() == at::kFloat, "rope tables must be fp32");
  TORCH_CHECK(cos.dim() == 2 && cos.size(1) == D / 2 && sin.sizes() == cos.sizes() && cos.is_contiguous() &&
                  sin.is_contiguous(), "rope tables must be contiguous fp32 [positions, D / 2]");
  c10::cuda::CUDAGuard guard(qkv.device());
  if (!qkv_splits) qkv = qkv.contiguous();
  positions = positions.contiguous();
  const int B = static_cast<int>(qkv_shape[0]), T = static_cast<int>(qkv_shape[1]);
  const CacheArg ca = cache_arg(k_cache, pages, B, "rope_store");
  const CacheArg cv = cache_arg(v_cache, pages, B, "rope_store");
  TORCH_CHECK(ca.pages.page_rows == cv.pages.page_rows && k_cache.sizes() == v_cache.sizes(),
              "rope_store: K and V caches must share a layout");
  TORCH_CHECK(qkv_shape.size() == 3 && qkv_shape[2] == (H + 2 * Hkv) * D, "qkv width mismatch");
  auto q = at::empty({B, T, H, D}, qkv.options().dtype(at::kBFloat16));
  const int rc = ecz::launch_rope_store(
      qkv_splits ? nullptr : qkv.data_ptr(), positions.data_ptr<int>(), cos.data_ptr<float>(), sin.data_ptr<float>(), q.data_ptr(),
      k_cache.data_ptr(), v_cache.data_ptr(), kv_len.data_ptr<int>(), n_new.data_ptr<int>(),
      q_norm.has_value() ? q_norm->data_ptr() : nullptr, k_norm.has_value() ? k_norm->data_ptr() : nullptr,
      static_cast<float>(eps), B, T, static_cast<int>(H), static_cast<int>(Hkv), static_cast<int>(D),
      ca.S, static_cast<int>(q_offset), at::cuda::getCurrentCUDAStream(),
      fp8 ? k_scale->data_ptr<float>() : nullptr, fp8 ? v_scale->data_ptr<float>() : nullptr,
      qkv_splits ? qkv.data_ptr<float>() : nullptr, qkv_splits, ca.pages, static_cast<int>(cos.size(0)),
      status_word(qkv.device()));
  TORCH_CHECK(rc == 0, "rope_store: unsupported head_dim ", D);
  return q;
}

Tensor attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor kv_len, Tensor n_new, c10::optional<Tensor> mask,
                 double scale, int64_t q_offset, c10::optional<Tensor> trace, c10::optional<Tensor> k_scale,
                 c10::optional<Tensor> v_scale, c10::optional<Tensor> keep, c10::optional<Tensor> lse_out,
                 c10::optional<Tensor> kivi, c10::optional<Tensor> kivi_chunks, int64_t kivi_bits, int64_t tail,
                 double softcap, c10::optional<Tensor> sinks, int64_t window, c10::optional<Tensor> pages) {
  CHECK_CUDA(q);
  CHECK_BF16(q);
  TORCH_CHECK(q.dim() == 4 && (q.size(3) == 128 || q.size(3) == 64 || q.size(3) == 256) && k_cache.dim() == 4,
              "attention: head_dim must be 64, 128 or 256");
  TORCH_CHECK(softcap >= 0.0 && window >= 0, "attention: softcap and window must be >= 0");
  if (sinks.has_value()) {
    CHECK_ON(*sinks, q);
    TORCH_CHECK(sinks->scalar_type() == at::kFloat && sinks->is_contiguous() && sinks->numel() == q.size(2),
                "attention: sinks must be fp32 [H] (one logit per query head)");
  }
  if (window > 0) {
    TORCH_CHECK(!mask.has_value() || window > 64, "attention: a sliding window must exceed 64 positions in tree "
                "passes");
    TORCH_CHECK(tail == 0 || window > tail, "attention: a sliding window must exceed the exact tail");
  }
  TORCH_CHECK(tail >= 0 && tail <= 64, "attention: the exact tail covers 0 .. 64 positions");
  const bool fp8 = fp8_cache(k_cache, k_scale, v_scale, k_cache.size(1));
  TORCH_CHECK(v_cache.scalar_type() == k_cache.scalar_type(), "K and V caches must share a dtype");
  CHECK_I32(kv_len);
  CHECK_I32(n_new);
  CHECK_ON(kv_len, q);
  CHECK_ON(n_new, q);
  CHECK_ON(k_cache, q);
  CHECK_ON(v_cache, q);
  if (mask.has_value()) CHECK_ON(*mask, q);
  if (keep.has_value()) CHECK_ON(*keep, q);
  if (lse_out.has_value()) CHECK_ON(*lse_out, q);
  if (kivi.has_value()) CHECK_ON(*kivi, q);
  if (kivi_chunks.has_value()) CHECK_ON(*kivi_chunks, q);
  TORCH_CHECK(q.dim() == 4 && k_cache.dim() == 4, "attention expects q [B, T, H, D] and caches [B, Hkv, S, D]");
  c10::cuda::CUDAGuard guard(q.device());
  q = q.contiguous();
  const int B = static_cast<int>(q.size(0)), T = static_cast<int>(q.size(1)), H = static_cast<int>(q.size(2)),
            D = static_cast<int>(q.size(3));
  const CacheArg ck = cache_arg(k_cache, pages, B, "attention");
  const CacheArg cv = cache_arg(v_cache, pages, B, "attention");
  TORCH_CHECK(ck.pages.page_rows == cv.pages.page_rows && k_cache.sizes() == v_cache.sizes(),
              "attention: K and V caches must share a layout");
  if (!pages.has_value()) TORCH_CHECK(k_cache.size(0) == B, "attention: caches must have q's batch");
  const int Hkv = static_cast<int>(k_cache.size(1)), S = ck.S;
  const int64_t* mask_ptr = nullptr;
  Tensor m;
  if (mask.has_value()) {
    m = mask->contiguous();
    CHECK_I64(m);
    TORCH_CHECK(T <= 64, "tree masks cover at most 64 new tokens");
    mask_ptr = m.data_ptr<int64_t>();
  }
  if (keep.has_value()) {
    CHECK_I32(*keep);
    TORCH_CHECK(keep->is_contiguous() && keep->numel() == static_cast<int64_t>(B) * Hkv * (S / 32),
                "keep must be int32 [B, Hkv, S / 32] bit words");
  }
  if (kivi.has_value()) {
    TORCH_CHECK(kivi->scalar_type() == at::kByte && kivi->is_contiguous() && kivi_chunks.has_value(),
                "kivi storage must be contiguous uint8 with chunk counts");
    TORCH_CHECK(kivi->numel() == static_cast<int64_t>(B) * Hkv * (S / 128) * ecz::kivi_chunk_size(kivi_bits),
                "kivi storage must be [B, Hkv, S / 128, chunk bytes]");
    CHECK_I32(*kivi_chunks);
  }
  if (lse_out.has_value()) {
    TORCH_CHECK(lse_out->scalar_type() == at::kFloat && lse_out->is_contiguous() &&
                    lse_out->numel() == static_cast<int64_t>(B) * T * H,
                "lse_out must be fp32 [B, T, H]");
  }
  auto out = at::empty_like(q);
  if (tail > 0) TORCH_CHECK(T <= 64, "attention: the exact tail serves passes of at most 64 query tokens");
  TORCH_CHECK(k_cache.size(3) == D && v_cache.size(3) == D, "attention: caches must have q's head_dim");
  const ecz::AttnPlan plan = ecz::attention_plan(B, T, H, Hkv, S, num_sms(q.get_device()), tail > 0, D,
                                                 static_cast<int>(window));
  if (trace.has_value()) {  // sixteen int64 stamps per CTA
    CHECK_ON(*trace, q);
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                    trace->numel() >= static_cast<int64_t>(B) * Hkv * plan.m_tiles * plan.splits * 16,
                "attention: trace must be a contiguous int64 tensor of at least 16 stamps per CTA");
  }
  ecz::AttnOpts opts;
  opts.softcap = static_cast<float>(softcap);
  opts.sinks = sinks.has_value() ? sinks->data_ptr<float>() : nullptr;
  opts.window = static_cast<int>(window);
  Tensor ws;
  if (plan.ws_floats > 0) ws = at::empty({plan.ws_floats}, q.options().dtype(at::kFloat));
  const CUtensorMap* tk = fp8 ? tensor_map_ex(k_cache.data_ptr(), 1, ck.rows, D, D, D, 128, 0)
                              : tensor_map(k_cache.data_ptr(), ck.rows, D, D, 128);
  const CUtensorMap* tv = fp8 ? tensor_map_ex(v_cache.data_ptr(), 1, cv.rows, D, D, D, 128, 0)
                              : tensor_map(v_cache.data_ptr(), cv.rows, D, D, 128);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int rc = ecz::launch_attention(q.data_ptr(), tk, tv, out.data_ptr(),
                                       plan.ws_floats > 0 ? ws.data_ptr<float>() : nullptr, kv_len.data_ptr<int>(),
                                       n_new.data_ptr<int>(), mask_ptr, B, T, H, Hkv, D, S,
                                       static_cast<float>(scale), static_cast<int>(q_offset), plan,
                                       status_word(q.device()), stream,
                                       trace.has_value() ? reinterpret_cast<unsigned long long*>(
                                                               trace->data_ptr<int64_t>())
                                                         : nullptr,
                                       fp8 ? k_scale->data_ptr<float>() : nullptr,
                                       fp8 ? v_scale->data_ptr<float>() : nullptr,
                                       keep.has_value() ? reinterpret_cast<const uint32_t*>(keep->data_ptr<int>())
                                                        : nullptr,
                                       lse_out.has_value() ? lse_out->data_ptr<float>() : nullptr,
                                       kivi.has_value() ? kivi->data_ptr<uint8_t>() : nullptr,
                                       kivi.has_value() ? kivi_chunks->data_ptr<int>() : nullptr,
                                       static_cast<int>(kivi_bits), static_cast<int>(tail), k_cache.data_ptr(),
                                       v_cache.data_ptr(), opts, ck.pages);
  if (rc == -3) {
    const cudaError_t err = cudaGetLastError();  // clears the refused launch's error state
    TORCH_CHECK(false, "attention: a kernel launch was refused: ", cudaGetErrorString(err));
  }
  TORCH_CHECK(rc == 0, "attention: unsupported shape (head_dim 64, 128 or 256, fp8 and KIVI caches at 128, H "
              "divisible by H_kv)");
  return out;
}

Tensor glu_act(Tensor gu, int64_t act, double limit) {
  CHECK_CUDA(gu);
  c10::cuda::CUDAGuard guard(gu.device());
  gu = gu.contiguous();
  auto [splits, shape] = parts_of(gu);
  const int F2 = static_cast<int>(shape.back());
  int64_t numel = 1;
  for (auto d : shape) numel *= d;
  const int rows = static_cast<int>(numel / F2);
  shape.back() = F2 / 2;
  auto out = at::empty(shape, gu.options().dtype(at::kBFloat16));
  const int rc = ecz::launch_glu(splits ? nullptr : gu.data_ptr(), out.data_ptr(), rows, F2 / 2,
                                 at::cuda::getCurrentCUDAStream(), splits ? gu.data_ptr<float>() : nullptr, splits,
                                 static_cast<int>(act), static_cast<float>(limit));
  TORCH_CHECK(rc == 0, "glu: width must be a multiple of 16 and act 0 (SiLU), 1 (GELU tanh) or 2 (clamped SwiGLU)");
  return out;
}

Tensor silu_mul(Tensor gu) { return glu_act(gu, 0, 0.0); }

// MInference vertical-slash pattern -> keep bit words: cols [..., nv], offsets [..., ns] (int64, same leading shape)
Tensor vs_keep(Tensor cols, Tensor offsets, int64_t base, int64_t t, int64_t limit, int64_t S) {
  CHECK_CUDA(cols);
  CHECK_ON(offsets, cols);
  TORCH_CHECK(cols.scalar_type() == at::kLong && offsets.scalar_type() == at::kLong, "vs_keep: int64 indices");
  TORCH_CHECK(cols.dim() >= 1 && offsets.dim() == cols.dim() &&
                  cols.sizes().slice(0, cols.dim() - 1) == offsets.sizes().slice(0, offsets.dim() - 1),
              "vs_keep: cols [..., nv] and offsets [..., ns] with the same leading shape");
  c10::cuda::CUDAGuard guard(cols.device());
  cols = cols.contiguous();
  offsets = offsets.contiguous();
  const int nv = static_cast<int>(cols.size(-1)), ns = static_cast<int>(offsets.size(-1));
  int64_t rows64 = 1;
  for (int64_t d = 0; d + 1 < cols.dim(); ++d) rows64 *= cols.size(d);
  const int rows = static_cast<int>(rows64);
  auto shape = cols.sizes().vec();
  shape.back() = S / 32;
  auto keep = at::empty(shape, cols.options().dtype(at::kInt));
  if (rows == 0) return keep;
  const int rc = ecz::launch_vs_keep(cols.data_ptr<int64_t>(), nv, offsets.data_ptr<int64_t>(), ns,
                                     static_cast<int>(base), static_cast<int>(t), static_cast<int>(limit), rows,
                                     static_cast<int>(S), reinterpret_cast<uint32_t*>(keep.data_ptr<int>()),
                                     at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc != -3, "vs_keep: the kernel launch was refused: ", cudaGetErrorString(cudaGetLastError()));
  TORCH_CHECK(rc == 0, "vs_keep: S must be a multiple of 32 and at most 262144, got ", S);
  return keep;
}

// Block Walsh-Hadamard transform of the last dimension of a bf16 tensor (blocks of `block`, a power of two in
// [8, 8192] dividing the width), scaled by 1 / sqrt(block)
Tensor hadamard(Tensor x, int64_t block) {
  CHECK_CUDA(x);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "hadamard: bf16 input");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  if (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 != 0) x = x.clone();  // the kernel loads 16-byte vectors
  const int F = static_cast<int>(x.size(-1));
  const int rows = F ? static_cast<int>(x.numel() / F) : 0;
  auto out = at::empty_like(x);
  if (rows == 0) return out;
  const int rc = ecz::launch_hadamard(x.data_ptr(), out.data_ptr(), rows, F, static_cast<int>(block),
                                      at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc != -3, "hadamard: the kernel launch was refused: ", cudaGetErrorString(cudaGetLastError()));
  TORCH_CHECK(rc == 0, "hadamard: block ", block, " must be a power of two in [8, 8192] dividing the width ", F);
  return out;
}

// act(gate) * up of a fused [gate; up] projection (bf16, or split-K partials), rotated by the block Hadamard
// transform in the same kernel
Tensor glu_hadamard(Tensor gu, int64_t act, double limit, int64_t block) {
  CHECK_CUDA(gu);
  c10::cuda::CUDAGuard guard(gu.device());
  gu = gu.contiguous();
  if (reinterpret_cast<uintptr_t>(gu.data_ptr()) % 16 != 0) gu = gu.clone();  // 16-byte vector loads
  auto [splits, shape] = parts_of(gu);
  const int F2 = static_cast<int>(shape.back());
  int64_t numel = 1;
  for (auto d : shape) numel *= d;
  const int rows = F2 ? static_cast<int>(numel / F2) : 0;
  shape.back() = F2 / 2;
  auto out = at::empty(shape, gu.options().dtype(at::kBFloat16));
  if (rows == 0) return out;
  TORCH_CHECK(splits || gu.scalar_type() == at::kBFloat16, "glu_hadamard: bf16 input or fp32 split-K partials");
  TORCH_CHECK(act >= 0 && act <= 2, "glu_hadamard: act 0 (SiLU), 1 (GELU tanh) or 2 (clamped SwiGLU)");
  const int rc = ecz::launch_hadamard(splits ? nullptr : gu.data_ptr(), out.data_ptr(), rows, F2 / 2,
                                      static_cast<int>(block), at::cuda::getCurrentCUDAStream(), static_cast<int>(act),
                                      splits ? gu.data_ptr<float>() : nullptr, splits, static_cast<float>(limit));
  TORCH_CHECK(rc != -3, "glu_hadamard: the kernel launch was refused: ", cudaGetErrorString(cudaGetLastError()));
  TORCH_CHECK(rc == 0, "glu_hadamard: block ", block, " must be a power of two in [8, 8192] dividing the width ",
              F2 / 2);
  return out;
}

Tensor linear_bf16(Tensor x, Tensor w) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "linear expects x [M, K] and w [N, K]");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  w = w.contiguous();
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(w.size(0));
  auto y = at::empty({M, N}, x.options());
  if (M == 0) return y;
  const int bn = ecz::gemm_block_n(M);
  const int sms = num_sms(x.get_device());
  const long tiles = static_cast<long>((N + 127) / 128) * ((M + bn - 1) / bn);
  const CUtensorMap* tw = tensor_map(w.data_ptr(), N, K, K, 128);
  const CUtensorMap* tx = tensor_map(x.data_ptr(), M, K, K, bn);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int rc;
  if (tiles >= sms) {
    // enough tiles for every SM: persistent stream-K balances the last wave
    auto ws = at::empty({ecz::gemm_persistent_ws_floats(M, N, K, sms)}, x.options().dtype(at::kFloat));
    rc = ecz::launch_gemm_persistent(tw, tx, y.data_ptr(), ws.data_ptr<float>(), split_counters(x.device(), stream),
                                     M, N, K, sms, status_word(x.device()), stream);
  } else {
    // fewer tiles than SMs: split K over a cluster per tile, partials reduced over DSMEM
    rc = ecz::launch_gemm_cluster(tw, tx, y.data_ptr(), M, N, K, ecz::gemm_cluster_splits(M, N, K, sms),
                                  status_word(x.device()), stream);
  }
  TORCH_CHECK(rc == 0, "linear: K must be a multiple of 8 and N of 4");
  return y;
}

// Weight-only quantized linear: x [M, K] bf16, packed uint8 weights [N, K * bits / 8], scales (and int4 zeros)
// bf16 [K / group, N]; fmt 0 int4, 1 int8, 2 fp8-e4m3.
Tensor linear_wq(Tensor x, Tensor qweight, Tensor scales, c10::optional<Tensor> zeros, int64_t fmt, int64_t group,
                 int64_t splits) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(scales);
  TORCH_CHECK(qweight.scalar_type() == at::kByte, "qweight must be uint8");
  TORCH_CHECK(fmt == ecz::kWqInt4 || fmt == ecz::kWqInt8 || fmt == ecz::kWqFp8 || fmt == ecz::kWqInt2 ||
                  fmt == ecz::kWqMxfp4 || fmt == ecz::kWqNvfp4,
              "unknown weight format ", fmt);
  const bool fp4 = fmt == ecz::kWqMxfp4 || fmt == ecz::kWqNvfp4;
  const bool zp = fmt == ecz::kWqInt4 || fmt == ecz::kWqInt2;
  TORCH_CHECK(x.dim() == 2 && qweight.dim() == 2 && scales.dim() == 2, "linear_wq expects 2-D operands");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  TORCH_CHECK(qweight.is_contiguous() && scales.is_contiguous(), "packed weights and scales must be contiguous");
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(qweight.size(0));
  const int row_bytes = fmt == ecz::kWqInt4 || fp4 ? K / 2 : fmt == ecz::kWqInt2 ? K / 4 : K;
  TORCH_CHECK(qweight.size(1) == row_bytes, "qweight has ", qweight.size(1), " bytes per row, expected ", row_bytes);
  TORCH_CHECK(K % group == 0 && scales.size(0) == K / group && scales.size(1) == N, "scales must be [K / group, N]");
  if (fp4) {
    TORCH_CHECK(group == (fmt == ecz::kWqMxfp4 ? 32 : 16), "mxfp4 takes group 32, nvfp4 group 16");
    TORCH_CHECK(K % 64 == 0 && N % 8 == 0, "linear_wq: K must be a multiple of 64, N of 8");
  } else {
    TORCH_CHECK(K % 64 == 0 && group % 64 == 0 && N % 8 == 0,
                "linear_wq: K and group must be multiples of 64, N of 8");
  }
  Tensor z;
  if (zp) {
    TORCH_CHECK(zeros.has_value(), "int4 / int2 weights need zeros");
    z = zeros->contiguous();
    CHECK_BF16(z);
    TORCH_CHECK(z.sizes() == scales.sizes(), "zeros must match scales");
  }
  auto y = at::empty({M, N}, x.options());
  if (M == 0) return y;
  const int bn = ecz::gemm_block_n(M);
  ecz::WqMaps maps;
  maps.w = tensor_map_ex(qweight.data_ptr(), 1, N, row_bytes, row_bytes,
                         fmt == ecz::kWqInt4 || fp4 ? 32 : fmt == ecz::kWqInt2 ? 16 : 64, 128, 0);
  maps.s = tensor_map_ex(scales.data_ptr(), 2, K / group, N, static_cast<uint64_t>(N) * 2, 128,
                         fp4 ? 64 / static_cast<int>(group) : 1, 0);
  if (zp) maps.z = tensor_map_ex(z.data_ptr(), 2, K / group, N, static_cast<uint64_t>(N) * 2, 128, 1, 0);
  maps.x = tensor_map(x.data_ptr(), M, K, K, bn);
  const int sp = splits > 0 ? static_cast<int>(splits)
                            : ecz::gemm_wq_splits(M, N, K, static_cast<int>(fmt), num_sms(x.get_device()));
  const int rc = ecz::launch_gemm_wq(maps, y.data_ptr(), M, N, K, static_cast<int>(group), static_cast<int>(fmt), sp,
                                     status_word(x.device()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "linear_wq: launch failed (", rc, ")");
  return y;
}

// x @ w.T for a consumer that sums split-K partials itself (rmsnorm, silu_mul, rope_store): a bf16 [M, N] result
// when the GEMM needs no split, else the fp32 partials [splits, M, N] of the non-cluster split-K kernel (two CTAs
// per SM). Tiles wider than 64 tokens take the regular path.
Tensor linear_parts(Tensor x, Tensor w) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "linear_parts expects x [M, K] and w [N, K]");
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(w.size(0));
  const int bn = ecz::gemm_block_n(M);
  if (bn > 64 || M == 0) return linear_bf16(x, w);
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  w = w.contiguous();
  const int sms = num_sms(x.get_device());
  int splits = std::min(8, ecz::gemm_splits(M, N, K, 2 * sms));
  const int total_kb = (K + 63) / 64, kbps = (total_kb + splits - 1) / splits;
  splits = (total_kb + kbps - 1) / kbps;  // the launcher drops empty splits the same way
  const CUtensorMap* tw = tensor_map(w.data_ptr(), N, K, K, 128);
  const CUtensorMap* tx = tensor_map(x.data_ptr(), M, K, K, bn);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  Tensor out = splits > 1 ? at::empty({splits, M, N}, x.options().dtype(at::kFloat)) : at::empty({M, N}, x.options());
  const int rc = ecz::launch_gemm_bf16(tw, tx, splits > 1 ? nullptr : out.data_ptr(),
                                       splits > 1 ? out.data_ptr<float>() : nullptr, M, N, K, splits,
                                       status_word(x.device()), stream, nullptr, nullptr, 3);
  TORCH_CHECK(rc == 0, "linear_parts: launch failed (", rc, ")");
  return out;
}

// Top-k routing of router logits [T, E] (bf16): expert ids [T, k] and renormalised weights [T, k] (fp32), each
// pair's row in expert order pos [T, k] and the expert offsets [E + 1] (int32).
std::tuple<Tensor, Tensor, Tensor, Tensor> moe_route(Tensor logits, int64_t k) {
  CHECK_CUDA(logits);
  CHECK_BF16(logits);
  c10::cuda::CUDAGuard guard(logits.device());
  logits = logits.contiguous();
  const int T = static_cast<int>(logits.size(0)), E = static_cast<int>(logits.size(1));
  auto i32 = logits.options().dtype(at::kInt);
  auto ids = at::empty({T, k}, i32), pos = at::empty({T, k}, i32), offsets = at::empty({E + 1}, i32);
  auto w = at::empty({T, k}, logits.options().dtype(at::kFloat));
  const int rc = ecz::launch_moe_route(logits.data_ptr(), T, E, static_cast<int>(k), ids.data_ptr<int>(),
                                       w.data_ptr<float>(), pos.data_ptr<int>(), offsets.data_ptr<int>(),
                                       at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "moe_route: at most 64 experts and top-8");
  return {ids, w, pos, offsets};
}

Tensor moe_gather(Tensor x, Tensor pos) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_I32(pos);
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  const int T = static_cast<int>(pos.size(0)), k = static_cast<int>(pos.size(1)), H = static_cast<int>(x.size(1));
  auto xs = at::empty({T * k, H}, x.options());
  TORCH_CHECK(ecz::launch_moe_gather(x.data_ptr(), pos.data_ptr<int>(), xs.data_ptr(), T, k, H,
                                     at::cuda::getCurrentCUDAStream()) == 0, "moe_gather: H % 8 != 0");
  return xs;
}

Tensor moe_combine(Tensor y, Tensor pos, Tensor w) {
  CHECK_CUDA(y);
  CHECK_BF16(y);
  c10::cuda::CUDAGuard guard(y.device());
  const int T = static_cast<int>(pos.size(0)), k = static_cast<int>(pos.size(1)), H = static_cast<int>(y.size(1));
  auto out = at::empty({T, H}, y.options());
  TORCH_CHECK(ecz::launch_moe_combine(y.contiguous().data_ptr(), pos.data_ptr<int>(), w.data_ptr<float>(),
                                      out.data_ptr(), T, k, H, at::cuda::getCurrentCUDAStream()) == 0,
              "moe_combine failed");
  return out;
}

// Grouped expert GEMM: rows offsets[e] .. offsets[e + 1] of xs [R, K] times expert e of w [E, N, K].
Tensor linear_grouped(Tensor xs, Tensor w, Tensor offsets) {
  CHECK_CUDA(xs);
  CHECK_BF16(xs);
  CHECK_BF16(w);
  CHECK_I32(offsets);
  TORCH_CHECK(w.dim() == 3 && xs.dim() == 2 && xs.size(1) == w.size(2), "linear_grouped: xs [R, K], w [E, N, K]");
  c10::cuda::CUDAGuard guard(xs.device());
  xs = xs.contiguous();
  w = w.contiguous();
  const int R = static_cast<int>(xs.size(0)), K = static_cast<int>(xs.size(1));
  const int E = static_cast<int>(w.size(0)), N = static_cast<int>(w.size(1));
  auto y = at::empty({R, N}, xs.options());
  if (R == 0) return y;
  const CUtensorMap* tw = tensor_map(w.data_ptr(), static_cast<uint64_t>(E) * N, K, K, 128);
  const CUtensorMap* tx = tensor_map(xs.data_ptr(), R, K, K, ecz::grouped_block_n(R, E));
  const int rc = ecz::launch_gemm_grouped(tw, tx, y.data_ptr(), offsets.data_ptr<int>(), E, R, N, K,
                                          status_word(xs.device()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "linear_grouped: K must be a multiple of 64 and N of 8");
  return y;
}

// Block-scaled fp8 linear: x [M, K] bf16 is quantised per token and 128-wide K block, then multiplied with e4m3
// weight codes [N, K] (uint8) whose fp32 scales are [N / 128, K / 128].
Tensor linear_fp8(Tensor x, Tensor wq, Tensor sw, int64_t splits) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  TORCH_CHECK(wq.scalar_type() == at::kByte && sw.scalar_type() == at::kFloat, "fp8 weights: uint8 codes, fp32 scales");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(wq.size(0));
  TORCH_CHECK(wq.size(1) == K && K % 128 == 0 && N % 128 == 0, "linear_fp8: K and N must be multiples of 128");
  TORCH_CHECK(sw.size(0) == N / 128 && sw.size(1) == K / 128 && sw.is_contiguous(), "scales must be [N/128, K/128]");
  auto y = at::empty({M, N}, x.options());
  if (M == 0) return y;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto q = at::empty({M, K}, x.options().dtype(at::kByte));
  const int sx_stride = (M + 3) / 4 * 4;  // TMA rows must be 16-byte multiples
  auto sx = at::empty({K / 128, sx_stride}, x.options().dtype(at::kFloat));
  TORCH_CHECK(ecz::launch_act_quant_fp8(x.data_ptr(), q.data_ptr(), sx.data_ptr<float>(), M, K, sx_stride, stream) ==
                  0,
              "activation quantisation failed");
  const int bn = ecz::fp8_block_n(M);
  const int sms = num_sms(x.get_device());
  int sp = splits > 0 ? static_cast<int>(splits) : std::min(8, ecz::gemm_splits(M, N, K, bn <= 64 ? 2 * sms : sms));
  const int total_kb = K / 128, kbps = (total_kb + sp - 1) / sp;
  sp = (total_kb + kbps - 1) / kbps;
  const CUtensorMap* tw = tensor_map_ex(wq.data_ptr(), 1, N, K, K, 128, 128, 128);
  const CUtensorMap* tx = tensor_map_ex(q.data_ptr(), 1, M, K, K, 128, bn, 128);
  const CUtensorMap* ts = tensor_map_ex(sx.data_ptr(), 4, K / 128, M, static_cast<uint64_t>(sx_stride) * 4, bn, 1, 0);
  Tensor ws;
  if (sp > 1) ws = at::empty({static_cast<int64_t>(sp) * M * N}, x.options().dtype(at::kFloat));
  const int rc = ecz::launch_gemm_fp8(tw, tx, ts, sw.data_ptr<float>(), y.data_ptr(),
                                      sp > 1 ? ws.data_ptr<float>() : nullptr, M, N, K, sp, status_word(x.device()),
                                      stream);
  TORCH_CHECK(rc == 0, "linear_fp8: launch failed (", rc, ")");
  return y;
}

// Top-k log-probabilities of fp32 logit rows [..., V] and their (optionally draft-to-target mapped) ids.
std::tuple<Tensor, Tensor> topk_logp(Tensor logits, int64_t k, double floor_v, c10::optional<Tensor> d2t) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat, "topk_logp takes fp32 logits");
  c10::cuda::CUDAGuard guard(logits.device());
  logits = logits.contiguous();
  const int V = static_cast<int>(logits.size(-1));
  const int rows = static_cast<int>(logits.numel() / V);
  std::vector<int64_t> shape(logits.sizes().begin(), logits.sizes().end());
  shape.back() = k;
  auto vals = at::empty(shape, logits.options());
  auto ids = at::empty(shape, logits.options().dtype(at::kLong));
  if (d2t.has_value()) {
    CHECK_I64(*d2t);
    TORCH_CHECK(d2t->numel() == V, "d2t must have one entry per logit");
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int splits = rows <= 1024 ? ecz::topk_splits(rows, V, num_sms(logits.get_device())) : 1;
  Tensor ws;
  if (splits > 1) {
    ws = at::empty({static_cast<int64_t>(ecz::topk_workspace_bytes(rows, splits))}, logits.options().dtype(at::kByte));
  }
  const int rc = ecz::launch_topk_logp(logits.data_ptr<float>(), d2t.has_value() ? d2t->data_ptr<int64_t>() : nullptr,
                                       vals.data_ptr<float>(), ids.data_ptr<int64_t>(), rows, V, static_cast<int>(k),
                                       static_cast<float>(floor_v), stream, splits,
                                       splits > 1 ? ws.data_ptr() : nullptr,
                                       splits > 1 ? arrival_counters(logits.device(), stream, 0) : nullptr);
  TORCH_CHECK(rc == 0, "topk_logp: 1 <= k <= 16");
  return {vals, ids};
}

// 2:4 sparse linear: kept bf16 values [N, K / 2] and their positions [N / 2, K / 4] (uint8), expanded to dense
// tiles in shared memory by the weight-streaming GEMM.
Tensor linear_sp24(Tensor x, Tensor values, Tensor meta, int64_t splits) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(values);
  TORCH_CHECK(meta.scalar_type() == at::kByte, "2:4 positions must be uint8");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(values.size(0));
  TORCH_CHECK(values.size(1) == K / 2 && values.is_contiguous(), "values must be [N, K / 2]");
  TORCH_CHECK(meta.size(0) == N / 2 && meta.size(1) == K / 4 && meta.is_contiguous(), "positions must be [N/2, K/4]");
  TORCH_CHECK(K % 64 == 0 && N % 8 == 0, "linear_sp24: K must be a multiple of 64, N of 8");
  auto y = at::empty({M, N}, x.options());
  if (M == 0) return y;
  ecz::WqMaps maps;
  maps.w = tensor_map_ex(values.data_ptr(), 2, N, K / 2, static_cast<uint64_t>(K), 32, 128, 0);
  maps.s = tensor_map_ex(meta.data_ptr(), 1, N / 2, K / 4, static_cast<uint64_t>(K / 4), 16, 64, 0);
  maps.x = tensor_map(x.data_ptr(), M, K, K, ecz::gemm_block_n(M));
  const int sp = splits > 0 ? static_cast<int>(splits)
                            : ecz::gemm_wq_splits(M, N, K, ecz::kWqInt8, num_sms(x.get_device()));
  const int rc = ecz::launch_gemm_wq(maps, y.data_ptr(), M, N, K, K, ecz::kWqSp24, sp, status_word(x.device()),
                                     at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "linear_sp24: launch failed (", rc, ")");
  return y;
}

// Accumulate KV-eviction scores [B, Hkv, S] (fp32, in place) for the queries q [B, T, H, D] of a pass whose
// log2-domain log-sum-exp lse2 [B, T, H] came from attention(..., lse_out=).
void attention_scores(Tensor q, Tensor k_cache, Tensor kv_len, Tensor n_new, c10::optional<Tensor> mask,
                      Tensor lse2, Tensor scores, double scale, int64_t q_offset, c10::optional<Tensor> pages) {
  CHECK_CUDA(q);
  CHECK_BF16(q);
  CHECK_BF16(k_cache);
  TORCH_CHECK(q.dim() == 4 && q.size(3) == 128 && k_cache.dim() == 4, "attention_scores: head_dim must be 128");
  c10::cuda::CUDAGuard guard(q.device());
  q = q.contiguous();
  const int B = static_cast<int>(q.size(0)), T = static_cast<int>(q.size(1)), H = static_cast<int>(q.size(2));
  const CacheArg ck = cache_arg(k_cache, pages, B, "attention_scores");
  const int Hkv = static_cast<int>(k_cache.size(1)), S = ck.S;
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.is_contiguous() &&
                  scores.numel() == static_cast<int64_t>(B) * Hkv * S, "scores must be fp32 [B, Hkv, S]");
  TORCH_CHECK(lse2.scalar_type() == at::kFloat && lse2.numel() == static_cast<int64_t>(B) * T * H, "lse2 [B, T, H]");
  CHECK_ON(k_cache, q);
  CHECK_ON(scores, q);
  CHECK_ON(lse2, q);
  CHECK_ON(kv_len, q);
  CHECK_ON(n_new, q);
  if (mask.has_value()) CHECK_ON(*mask, q);
  Tensor m;
  if (mask.has_value()) {
    m = mask->contiguous();
    CHECK_I64(m);
  }
  const CUtensorMap* tk = tensor_map(k_cache.data_ptr(), ck.rows, 128, 128, 128);
  const int rc = ecz::launch_attention_scores(q.data_ptr(), tk, lse2.contiguous().data_ptr<float>(),
                                              scores.data_ptr<float>(), kv_len.data_ptr<int>(), n_new.data_ptr<int>(),
                                              mask.has_value() ? m.data_ptr<int64_t>() : nullptr, B, T, H, Hkv, 128, S,
                                              static_cast<float>(scale), static_cast<int>(q_offset),
                                              status_word(q.device()), at::cuda::getCurrentCUDAStream(), ck.pages);
  TORCH_CHECK(rc == 0, "attention_scores: unsupported shape");
}

void kivi_quantize(Tensor cache, Tensor kivi, Tensor kv_len, Tensor chunks, int64_t bits, int64_t residual,
                   int64_t max_new, c10::optional<Tensor> pages) {
  CHECK_CUDA(cache);
  CHECK_BF16(cache);
  CHECK_I32(kv_len);
  CHECK_I32(chunks);
  CHECK_CUDA(cache);
  CHECK_ON(kivi, cache);
  CHECK_ON(kv_len, cache);
  CHECK_ON(chunks, cache);
  const WholeCache w = whole_cache(cache, pages, "kivi_quantize");
  c10::cuda::CUDAGuard guard(cache.device());
  const int L = w.L, B = w.B, Hkv = w.Hkv, S = w.S, D = w.D;
  TORCH_CHECK(kivi.scalar_type() == at::kByte && kivi.is_contiguous() &&
                  kivi.numel() == static_cast<int64_t>(L) * B * Hkv * (S / 128) * ecz::kivi_chunk_size(bits),
              "kivi storage must be [L, B, Hkv, S / 128, chunk bytes]");
  const int rc = ecz::launch_kivi_quantize(cache.data_ptr(), kivi.data_ptr(), kv_len.data_ptr<int>(),
                                           chunks.data_ptr<int>(), L, B, Hkv, S, D, static_cast<int>(bits),
                                           static_cast<int>(residual), static_cast<int>(max_new),
                                           at::cuda::getCurrentCUDAStream(), w.layout);
  TORCH_CHECK(rc == 0, "kivi_quantize: head_dim 128, 2 or 4 bits");
}

// Explicit GEMM variant (tuning and benchmarks): mode 1 cluster split-K (DSMEM reduction), 2 split-K through a
// global fp32 workspace reduced by the tile's last CTA, 3 persistent stream-K; splits <= 0 picks the default.
Tensor linear_variant(Tensor x, Tensor w, int64_t mode, int64_t splits) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "linear expects x [M, K] and w [N, K]");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  w = w.contiguous();
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(w.size(0));
  auto y = at::empty({M, N}, x.options());
  if (M == 0) return y;
  const int bn = ecz::gemm_block_n(M);
  const int sms = num_sms(x.get_device());
  const CUtensorMap* tw = tensor_map(w.data_ptr(), N, K, K, 128);
  const CUtensorMap* tx = tensor_map(x.data_ptr(), M, K, K, bn);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int rc = -1;
  if (mode == 1) {
    const int sp = splits > 0 ? static_cast<int>(splits) : ecz::gemm_cluster_splits(M, N, K, sms);
    rc = ecz::launch_gemm_cluster(tw, tx, y.data_ptr(), M, N, K, sp, status_word(x.device()), stream);
  } else if (mode == 2) {
    const int sp = splits > 0 ? static_cast<int>(splits) : ecz::gemm_splits(M, N, K, sms);
    auto ws = at::empty({static_cast<int64_t>(sp) * M * N}, x.options().dtype(at::kFloat));
    rc = ecz::launch_gemm_bf16(tw, tx, y.data_ptr(), ws.data_ptr<float>(), M, N, K, sp, status_word(x.device()),
                               stream, split_counters(x.device(), stream));
  } else if (mode >= 4 && mode <= 6) {
    // 4: two CTAs per SM, fp32 partials left in a workspace (GEMM part only); 5: same + separate reduce kernel;
    // 6: two CTAs per SM with the in-kernel last-CTA reduction
    const int sp = splits > 0 ? static_cast<int>(splits) : ecz::gemm_splits(M, N, K, 2 * sms);
    auto ws = at::empty({static_cast<int64_t>(sp) * M * N}, x.options().dtype(at::kFloat));
    rc = ecz::launch_gemm_bf16(tw, tx, y.data_ptr(), ws.data_ptr<float>(), M, N, K, sp, status_word(x.device()),
                               stream, mode == 6 ? split_counters(x.device(), stream) : nullptr, nullptr,
                               mode == 4 ? 3 : 1);
  } else if (mode == 3) {
    auto ws = at::empty({ecz::gemm_persistent_ws_floats(M, N, K, sms)}, x.options().dtype(at::kFloat));
    rc = ecz::launch_gemm_persistent(tw, tx, y.data_ptr(), ws.data_ptr<float>(), split_counters(x.device(), stream),
                                     M, N, K, sms, status_word(x.device()), stream);
  }
  TORCH_CHECK(rc == 0, "linear_variant: mode ", mode, " failed (", rc, ")");
  return y;
}

int64_t gemm_cluster_capacity(int64_t M, int64_t splits) {
  return ecz::gemm_cluster_capacity(static_cast<int>(M), static_cast<int>(splits));
}

Tensor argmax(Tensor x) {
  CHECK_CUDA(x);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "argmax takes bf16 or fp32");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  const int V = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / V);
  auto out = at::empty({rows}, x.options().dtype(at::kLong));
  const int slices = ecz::argmax_slices(rows, V);
  auto part = at::empty({2 * static_cast<int64_t>(rows) * slices}, x.options().dtype(at::kFloat));
  ecz::launch_argmax(x.data_ptr(), x.scalar_type() == at::kBFloat16, out.data_ptr<int64_t>(),
                     part.data_ptr<float>(), reinterpret_cast<int*>(part.data_ptr<float>() + rows * slices), rows, V,
                     at::cuda::getCurrentCUDAStream());
  return out;
}

std::tuple<Tensor, Tensor, Tensor> greedy_accept(Tensor tokens, Tensor parents, Tensor pred,
                                                 c10::optional<Tensor> ok) {
  CHECK_CUDA(tokens);
  CHECK_I64(tokens);
  CHECK_I64(parents);
  CHECK_I64(pred);
  CHECK_ON(parents, tokens);
  CHECK_ON(pred, tokens);
  if (ok.has_value()) CHECK_ON(*ok, tokens);
  c10::cuda::CUDAGuard guard(tokens.device());
  tokens = tokens.contiguous();
  parents = parents.contiguous();
  pred = pred.contiguous();
  const int B = static_cast<int>(tokens.size(0)), T = static_cast<int>(tokens.size(1));
  auto n_acc = at::empty({B}, tokens.options().dtype(at::kInt));
  auto path = at::empty({B, T}, tokens.options().dtype(at::kInt));
  auto out = at::empty({B, T}, tokens.options());
  Tensor okc;
  if (ok.has_value()) {
    okc = ok->to(at::kByte).contiguous();
    TORCH_CHECK(okc.numel() == static_cast<int64_t>(B) * T, "ok must be [B, T]");
  }
  const int rc = ecz::launch_greedy_accept(tokens.data_ptr<int64_t>(), parents.data_ptr<int64_t>(),
                                           pred.data_ptr<int64_t>(), ok.has_value() ? okc.data_ptr<uint8_t>() : nullptr,
                                           n_acc.data_ptr<int>(), path.data_ptr<int>(), out.data_ptr<int64_t>(), B, T,
                                           at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "greedy_accept: at most 64 tree nodes");
  return {n_acc, path, out};
}

void kv_compact(Tensor cache, Tensor kv_len, Tensor path, Tensor n_acc, c10::optional<Tensor> pages) {
  CHECK_CUDA(cache);
  TORCH_CHECK(cache.element_size() == 2 || cache.element_size() == 1, "cache must be bf16 or fp8");
  CHECK_I32(kv_len);
  CHECK_I32(path);
  CHECK_I32(n_acc);
  CHECK_ON(kv_len, cache);
  CHECK_ON(path, cache);
  CHECK_ON(n_acc, cache);
  const WholeCache w = whole_cache(cache, pages, "kv_compact");
  c10::cuda::CUDAGuard guard(cache.device());
  path = path.contiguous();
  const int T = static_cast<int>(path.size(1));
  const int max_depth = std::max(1, T - 1);
  const int rc = ecz::launch_kv_compact(cache.data_ptr(), kv_len.data_ptr<int>(), path.data_ptr<int>(),
                                        n_acc.data_ptr<int>(), w.L, w.B, w.Hkv, w.S,
                                        w.D * static_cast<int>(cache.element_size()), T, std::min(max_depth, 64),
                                        at::cuda::getCurrentCUDAStream(), w.layout);
  TORCH_CHECK(rc == 0, "kv_compact: unsupported head_dim or path length");
}

Tensor sample(Tensor probs, Tensor u) {
  CHECK_CUDA(probs);
  TORCH_CHECK(probs.scalar_type() == at::kFloat && u.scalar_type() == at::kFloat, "sample takes fp32 probs and u");
  c10::cuda::CUDAGuard guard(probs.device());
  probs = probs.contiguous();
  const int V = static_cast<int>(probs.size(-1));
  const int rows = static_cast<int>(probs.numel() / V);
  TORCH_CHECK(u.numel() == rows, "one uniform per row");
  auto out = at::empty({rows}, probs.options().dtype(at::kLong));
  ecz::launch_sample(probs.data_ptr<float>(), u.contiguous().data_ptr<float>(), out.data_ptr<int64_t>(), rows, V,
                     at::cuda::getCurrentCUDAStream());
  return out;
}

std::tuple<Tensor, Tensor> rejection(Tensor p, Tensor q, Tensor drafts, Tensor u_acc, Tensor u_draw) {
  CHECK_CUDA(p);
  TORCH_CHECK(p.scalar_type() == at::kFloat && q.scalar_type() == at::kFloat, "p and q must be fp32");
  CHECK_I64(drafts);
  CHECK_ON(q, p);
  CHECK_ON(drafts, p);
  c10::cuda::CUDAGuard guard(p.device());
  p = p.contiguous();
  q = q.contiguous();
  drafts = drafts.contiguous();
  const int B = static_cast<int>(drafts.size(0)), k = static_cast<int>(drafts.size(1));
  const int V = static_cast<int>(p.size(-1));
  TORCH_CHECK(p.numel() == static_cast<int64_t>(B) * (k + 1) * V && q.numel() == static_cast<int64_t>(B) * k * V,
              "p [B, k+1, V], q [B, k, V]");
  auto n_acc = at::empty({B}, drafts.options().dtype(at::kInt));
  auto out = at::empty({B, k + 1}, drafts.options());
  ecz::launch_rejection(p.data_ptr<float>(), q.data_ptr<float>(), drafts.data_ptr<int64_t>(),
                        u_acc.contiguous().data_ptr<float>(), u_draw.contiguous().data_ptr<float>(),
                        n_acc.data_ptr<int>(), out.data_ptr<int64_t>(), B, k, V, at::cuda::getCurrentCUDAStream());
  return {n_acc, out};
}

Tensor ngram(Tensor history, Tensor len, int64_t k, int64_t min_n, int64_t max_n, bool earliest) {
  CHECK_CUDA(history);
  CHECK_I64(history);
  CHECK_I32(len);
  c10::cuda::CUDAGuard guard(history.device());
  history = history.contiguous();
  const int B = static_cast<int>(history.size(0)), cap = static_cast<int>(history.size(1));
  auto drafts = at::empty({B, k}, history.options());
  ecz::launch_ngram(history.data_ptr<int64_t>(), len.contiguous().data_ptr<int>(), drafts.data_ptr<int64_t>(), B, cap,
                    static_cast<int>(k), static_cast<int>(min_n), static_cast<int>(max_n), earliest,
                    at::cuda::getCurrentCUDAStream());
  return drafts;
}

// ---- symmetric memory over CUDA IPC -------------------------------------------------------------------------
// symm_alloc(bytes) -> (device pointer, IPC handle bytes); symm_open(handle) -> peer pointer; symm_free(ptr).
std::tuple<int64_t, py::bytes> symm_alloc(int64_t bytes) {
  void* ptr = nullptr;
  TORCH_CHECK(cudaMalloc(&ptr, bytes) == cudaSuccess, "symm_alloc: cudaMalloc failed");
  TORCH_CHECK(cudaMemset(ptr, 0, bytes) == cudaSuccess, "symm_alloc: cudaMemset failed");
  cudaIpcMemHandle_t handle;
  TORCH_CHECK(cudaIpcGetMemHandle(&handle, ptr) == cudaSuccess, "symm_alloc: cudaIpcGetMemHandle failed");
  return {reinterpret_cast<int64_t>(ptr), py::bytes(reinterpret_cast<const char*>(&handle), sizeof(handle))};
}

int64_t symm_open(py::bytes handle_bytes) {
  std::string raw = handle_bytes;
  TORCH_CHECK(raw.size() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle");
  cudaIpcMemHandle_t handle;
  std::memcpy(&handle, raw.data(), sizeof(handle));
  void* ptr = nullptr;
  const cudaError_t err = cudaIpcOpenMemHandle(&ptr, handle, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(err == cudaSuccess, "symm_open: cudaIpcOpenMemHandle failed: ", cudaGetErrorString(err));
  return reinterpret_cast<int64_t>(ptr);
}

void symm_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }
void symm_free(int64_t ptr) { cudaFree(reinterpret_cast<void*>(ptr)); }
int64_t symm_control_bytes() { return static_cast<int64_t>(ecz::symm_control_bytes()); }

ecz::PeerPtrs peer_ptrs(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK(ptrs.size() <= static_cast<size_t>(ecz::kMaxPeers), "at most 8 peers");
  ecz::PeerPtrs p{};
  for (size_t i = 0; i < ptrs.size(); ++i) p.ptr[i] = reinterpret_cast<void*>(ptrs[i]);
  return p;
}

// ---- activation sparsity (act_sparse.cu) ------------------------------------------------------------------------
// sparsify(x) @ W^T for x [M <= 16, K] and the transposed weight wt [K, N]: only the rows of wt whose input column
// some row keeps (|x| > threshold; no threshold: x != 0) are read.
Tensor colsparse_linear(Tensor x, Tensor wt, c10::optional<Tensor> threshold) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(wt);
  TORCH_CHECK(wt.dim() == 2 && wt.is_contiguous() && x.size(-1) == wt.size(0), "colsparse_linear: wt [K, N]");
  c10::cuda::CUDAGuard guard(x.device());
  const int K = static_cast<int>(wt.size(0)), N = static_cast<int>(wt.size(1));
  auto x2 = x.reshape({-1, K}).contiguous();
  const int M = static_cast<int>(x2.size(0));
  auto out = at::empty({M, N}, x.options());
  const float* thr = nullptr;
  if (threshold.has_value()) {
    TORCH_CHECK(threshold->scalar_type() == at::kFloat && threshold->numel() == 1 && threshold->is_cuda(),
                "colsparse_linear: threshold is a CUDA fp32 scalar");
    thr = threshold->data_ptr<float>();
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int splits = ecz::colsparse_splits(M, N, K, num_sms(x.get_device()));
  Tensor ws;
  if (splits > 8) ws = at::empty({splits / 8, M, N}, x.options().dtype(at::kFloat));
  const int rc = ecz::launch_colsparse_gemv(x2.data_ptr(), K, wt.data_ptr(), thr, out.data_ptr(),
                                            splits > 8 ? ws.data_ptr<float>() : nullptr,
                                            split_counters(x.device(), stream), M, N, K, splits, stream);
  TORCH_CHECK(rc == 0, "colsparse_linear: at most 16 rows and N a multiple of 8 (", rc, ")");
  auto sizes = x.sizes().vec();
  sizes.back() = N;
  return out.view(sizes);
}

// h = (silu(gate) * 1[keep]) * up of a gated MLP over x [M <= 16, H] with w_gate_up [2F, H] (gate rows first), only
// for kept channels. CATS: gate [M, F] given, keep = |silu(gate)| > threshold. Deja Vu: keep [M, F] (bool) given.
Tensor glu_rows(Tensor x, Tensor w_gate_up, c10::optional<Tensor> gate, c10::optional<Tensor> keep,
                c10::optional<Tensor> threshold) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w_gate_up);
  TORCH_CHECK(w_gate_up.dim() == 2 && w_gate_up.is_contiguous() && w_gate_up.size(1) == x.size(-1),
              "glu_rows: w_gate_up [2F, H]");
  c10::cuda::CUDAGuard guard(x.device());
  const int H = static_cast<int>(w_gate_up.size(1)), F = static_cast<int>(w_gate_up.size(0) / 2);
  auto x2 = x.reshape({-1, H}).contiguous();
  const int M = static_cast<int>(x2.size(0));
  auto h = at::empty({M, F}, x.options());
  const void* g = nullptr;
  int ld_gate = F;
  Tensor g2, k2;
  const uint8_t* kp = nullptr;
  if (keep.has_value()) {
    TORCH_CHECK(keep->numel() == static_cast<int64_t>(M) * F, "glu_rows: keep [M, F]");
    k2 = keep->reshape({M, F}).to(at::kByte).contiguous();
    kp = k2.data_ptr<uint8_t>();
  } else {
    TORCH_CHECK(gate.has_value() && threshold.has_value(), "glu_rows: CATS needs the gate output and a threshold");
    CHECK_BF16((*gate));
    g2 = gate->reshape({M, F}).contiguous();
    g = g2.data_ptr();
  }
  const float* thr = nullptr;
  if (threshold.has_value()) {
    TORCH_CHECK(threshold->scalar_type() == at::kFloat && threshold->numel() == 1 && threshold->is_cuda(),
                "glu_rows: threshold is a CUDA fp32 scalar");
    thr = threshold->data_ptr<float>();
  }
  const int rc = ecz::launch_glu_rows(x2.data_ptr(), H, w_gate_up.data_ptr(), g, ld_gate, kp, thr, h.data_ptr(), M, F,
                                      H, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "glu_rows: at most 16 rows and H a multiple of 8");
  auto sizes = x.sizes().vec();
  sizes.back() = F;
  return h.view(sizes);
}

// ---- draft trees (tree.cu) -------------------------------------------------------------------------------------
// One depth of a dynamic-tree expansion (see tree.cu); every tensor is updated in place.
void tree_expand(Tensor c_vals, Tensor c_ids, Tensor f_scores, Tensor f_cand, Tensor f_tokens, Tensor parent_fwd,
                 Tensor fwd_bits, Tensor origin, Tensor bits_next, Tensor cand_tokens, Tensor cand_scores,
                 Tensor cand_parents, int64_t d, bool next) {
  CHECK_CUDA(c_vals);
  TORCH_CHECK(c_vals.scalar_type() == at::kFloat && f_scores.scalar_type() == at::kFloat &&
                  cand_scores.scalar_type() == at::kFloat, "tree_expand: fp32 scores");
  for (const Tensor* t : {&c_ids, &f_cand, &f_tokens, &parent_fwd, &fwd_bits, &origin, &bits_next, &cand_tokens,
                          &cand_parents}) {
    TORCH_CHECK(t->scalar_type() == at::kLong && t->is_contiguous(), "tree_expand: contiguous int64 index tensors");
    CHECK_ON(*t, c_vals);
  }
  CHECK_ON(f_scores, c_vals);
  CHECK_ON(cand_scores, c_vals);
  TORCH_CHECK(c_vals.is_contiguous() && f_scores.is_contiguous() && cand_scores.is_contiguous(),
              "tree_expand: contiguous scores");
  c10::cuda::CUDAGuard guard(c_vals.device());
  const int B = static_cast<int>(f_scores.size(0)), k = static_cast<int>(f_scores.size(1));
  TORCH_CHECK(c_vals.numel() == static_cast<int64_t>(B) * k * k, "tree_expand: c_vals [B, k, k]");
  const int rc = ecz::launch_tree_expand(
      c_vals.data_ptr<float>(), c_ids.data_ptr<int64_t>(), f_scores.data_ptr<float>(), f_cand.data_ptr<int64_t>(),
      f_tokens.data_ptr<int64_t>(), parent_fwd.data_ptr<int64_t>(), fwd_bits.data_ptr<int64_t>(),
      origin.data_ptr<int64_t>(), bits_next.data_ptr<int64_t>(), cand_tokens.data_ptr<int64_t>(),
      cand_scores.data_ptr<float>(), cand_parents.data_ptr<int64_t>(), B, k, static_cast<int>(d),
      static_cast<int>(cand_tokens.size(1)), static_cast<int>(fwd_bits.size(1)), next,
      at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "tree_expand: k <= 16 and (d + 1) k <= 64");
}

// Ancestor bits [B, T] int64 and positions kv_len + depth [B, T] int32 of a verified tree given by its parents.
std::tuple<Tensor, Tensor> tree_layout(Tensor parents, Tensor kv_len) {
  CHECK_CUDA(parents);
  CHECK_ON(kv_len, parents);
  CHECK_I64(parents);
  CHECK_I32(kv_len);
  TORCH_CHECK(parents.dim() == 2 && parents.size(1) >= 1 && parents.size(1) <= 64, "tree_layout: parents [B, T <= 64]");
  c10::cuda::CUDAGuard guard(parents.device());
  parents = parents.contiguous();
  const int B = static_cast<int>(parents.size(0)), T = static_cast<int>(parents.size(1));
  TORCH_CHECK(kv_len.numel() == B && kv_len.is_contiguous(), "tree_layout: kv_len [B]");
  auto bits = at::empty({B, T}, parents.options());
  auto pos = at::empty({B, T}, parents.options().dtype(at::kInt));
  const int rc = ecz::launch_tree_layout(parents.data_ptr<int64_t>(), kv_len.data_ptr<int>(), bits.data_ptr<int64_t>(),
                                         pos.data_ptr<int>(), B, T, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "tree_layout: launch failed");
  return {bits, pos};
}

std::tuple<Tensor, Tensor> tree_select(Tensor cand_tokens, Tensor cand_scores, Tensor cand_parents, int64_t k,
                                       int64_t total) {
  CHECK_CUDA(cand_tokens);
  CHECK_ON(cand_scores, cand_tokens);
  CHECK_ON(cand_parents, cand_tokens);
  TORCH_CHECK(cand_tokens.scalar_type() == at::kLong && cand_parents.scalar_type() == at::kLong &&
                  cand_scores.scalar_type() == at::kFloat, "tree_select: int64 tokens / parents, fp32 scores");
  c10::cuda::CUDAGuard guard(cand_tokens.device());
  cand_tokens = cand_tokens.contiguous();
  cand_scores = cand_scores.contiguous();
  cand_parents = cand_parents.contiguous();
  const int B = static_cast<int>(cand_tokens.size(0)), N = static_cast<int>(cand_tokens.size(1));
  auto tokens = at::empty({B, total}, cand_tokens.options());
  auto parents = at::empty({B, total}, cand_tokens.options());
  const int rc = ecz::launch_tree_select(cand_tokens.data_ptr<int64_t>(), cand_scores.data_ptr<float>(),
                                         cand_parents.data_ptr<int64_t>(), B, N, static_cast<int>(k),
                                         static_cast<int>(total), tokens.data_ptr<int64_t>(),
                                         parents.data_ptr<int64_t>(), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "tree_select: 1 <= total <= candidates <= 4096");
  return {tokens, parents};
}

// ---- binary factors (binary.cu) ---------------------------------------------------------------------------------
// x [M <= 16, K] fp32 times the sign matrix bits [N, ceil(K / 32)] (int32 words, bit set = -1) -> [M, N] fp32.
Tensor sign_matvec(Tensor bits, Tensor x) {
  CHECK_CUDA(x);
  TORCH_CHECK(x.scalar_type() == at::kFloat && bits.scalar_type() == at::kInt, "sign_matvec: fp32 x, int32 bits");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  bits = bits.contiguous();
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(bits.size(0));
  TORCH_CHECK(bits.size(1) == (K + 31) / 32, "sign_matvec: bits [N, ceil(K / 32)]");
  auto out = at::empty({M, N}, x.options());
  const int rc = ecz::launch_sign_matvec(reinterpret_cast<const uint32_t*>(bits.data_ptr<int>()), x.data_ptr<float>(),
                                         out.data_ptr<float>(), M, N, K, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "sign_matvec: at most 16 rows");
  return out;
}

// ---- expert parallelism over NVLink peer memory (ep.cu) ---------------------------------------------------------
int64_t ep_buffer_bytes(int64_t world, int64_t experts_local, int64_t cap, int64_t hidden, int64_t ret_rows) {
  return ecz::ep_layout(static_cast<int>(world), static_cast<int>(experts_local), static_cast<int>(cap),
                        static_cast<int>(hidden), static_cast<int>(ret_rows)).bytes;
}

// One expert-parallel MoE MLP: xs [T k, H] are this rank's routed rows in global expert order (moe_gather), offsets
// [E + 1] the global expert offsets, pos / w [T, k] each pair's row and weight; w_gate_up [E_l, 2F, H] and w_down
// [E_l, H, F] this rank's experts. Dispatch, the two grouped GEMMs, combine and the weighted sum run on the device.
Tensor ep_moe(Tensor xs, Tensor offsets, Tensor pos, Tensor w, Tensor w_gate_up, Tensor w_down,
              std::vector<int64_t> ptrs, int64_t rank, int64_t cap, int64_t ret_rows) {
  CHECK_CUDA(xs);
  CHECK_BF16(xs);
  CHECK_BF16(w_gate_up);
  CHECK_BF16(w_down);
  CHECK_I32(offsets);
  CHECK_I32(pos);
  TORCH_CHECK(w.scalar_type() == at::kFloat, "ep_moe: fp32 routing weights");
  CHECK_ON(offsets, xs);
  CHECK_ON(pos, xs);
  CHECK_ON(w, xs);
  CHECK_ON(w_gate_up, xs);
  CHECK_ON(w_down, xs);
  c10::cuda::CUDAGuard guard(xs.device());
  xs = xs.contiguous();
  const int world = static_cast<int>(ptrs.size());
  const int El = static_cast<int>(w_gate_up.size(0)), F2 = static_cast<int>(w_gate_up.size(1));
  const int H = static_cast<int>(xs.size(1)), T = static_cast<int>(pos.size(0)), k = static_cast<int>(pos.size(1));
  TORCH_CHECK(offsets.numel() == static_cast<int64_t>(world) * El + 1, "ep_moe: offsets must cover world x E_l");
  TORCH_CHECK(w_gate_up.size(2) == H && w_down.size(0) == El && w_down.size(1) == H && w_down.size(2) * 2 == F2,
              "ep_moe: expert weight shapes");
  TORCH_CHECK(xs.size(0) == static_cast<int64_t>(T) * k && T * k <= cap && T * k <= ret_rows,
              "ep_moe: more routed rows than the buffers hold");
  const ecz::EpLayout L = ecz::ep_layout(world, El, static_cast<int>(cap), H, static_cast<int>(ret_rows));
  const ecz::PeerPtrs peers = peer_ptrs(ptrs);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  unsigned* status = status_word(xs.device());
  auto out = at::empty({T, H}, xs.options());
  const int G = world * El, R = world * static_cast<int>(cap), F = F2 / 2;
  auto seg = at::empty({3, G}, offsets.options());
  int* s0 = seg.data_ptr<int>();
  TORCH_CHECK(ecz::launch_ep_dispatch(xs.data_ptr(), offsets.data_ptr<int>(), peers, L, static_cast<int>(rank),
                                      T * k, stream) == 0, "ep_moe: dispatch launch failed");
  TORCH_CHECK(ecz::launch_ep_segments(peers, L, static_cast<int>(rank), s0, s0 + G, s0 + 2 * G, status, stream) == 0,
              "ep_moe: at most 128 (rank, expert) segments");
  void* recv = static_cast<uint8_t*>(reinterpret_cast<void*>(ptrs[rank])) + L.recv_off;
  const int bn = ecz::grouped_block_n(static_cast<int>(cap), G);
  auto gu = at::empty({R, F2}, xs.options());
  w_gate_up = w_gate_up.contiguous();
  w_down = w_down.contiguous();
  const CUtensorMap* tw1 = tensor_map(w_gate_up.data_ptr(), static_cast<uint64_t>(El) * F2, H, H, 128);
  const CUtensorMap* tx1 = tensor_map(recv, R, H, H, bn);
  TORCH_CHECK(ecz::launch_gemm_segments(tw1, tx1, gu.data_ptr(), s0, s0 + G, s0 + 2 * G, G, static_cast<int>(cap), F2,
                                        H, status, stream) == 0, "ep_moe: H must be a multiple of 64");
  auto a = at::empty({R, F}, xs.options());
  TORCH_CHECK(ecz::launch_silu_mul(gu.data_ptr(), a.data_ptr(), R, F, stream) == 0, "ep_moe: silu_mul failed");
  auto y = at::empty({R, H}, xs.options());
  const CUtensorMap* tw2 = tensor_map(w_down.data_ptr(), static_cast<uint64_t>(El) * H, F, F, 128);
  const CUtensorMap* tx2 = tensor_map(a.data_ptr(), R, F, F, bn);
  TORCH_CHECK(ecz::launch_gemm_segments(tw2, tx2, y.data_ptr(), s0, s0 + G, s0 + 2 * G, G, static_cast<int>(cap), H,
                                        F, status, stream) == 0, "ep_moe: F must be a multiple of 64");
  TORCH_CHECK(ecz::launch_ep_combine(y.data_ptr(), s0, s0 + G, peers, L, static_cast<int>(rank), stream) == 0,
              "ep_moe: combine launch failed");
  TORCH_CHECK(ecz::launch_ep_finish(peers, L, static_cast<int>(rank), pos.data_ptr<int>(), w.data_ptr<float>(),
                                    out.data_ptr(), T, k, status, stream) == 0, "ep_moe: finish launch failed");
  return out;
}

// Row-parallel GEMM whose output tiles go straight into every peer's slot (tensor-parallel push mode).
void linear_push(Tensor x, Tensor w, std::vector<int64_t> ptrs, int64_t rank, int64_t parity, int64_t slot_elems) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "linear_push expects x [M, K] and w [N, K]");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  w = w.contiguous();
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(w.size(0));
  TORCH_CHECK(static_cast<long>(M) * N <= slot_elems, "linear_push: output larger than the slot");
  const int sms = num_sms(x.get_device());
  const int splits = ecz::gemm_cluster_splits(M, N, K, sms);
  ecz::PeerOut peer{};
  peer.ptrs = peer_ptrs(ptrs);
  peer.world = static_cast<int>(ptrs.size());
  peer.rank = static_cast<int>(rank);
  peer.parity = static_cast<int>(parity);
  peer.slot_elems = slot_elems;
  peer.control_bytes = static_cast<long>(ecz::symm_control_bytes());
  const CUtensorMap* tw = tensor_map(w.data_ptr(), N, K, K, 128);
  const CUtensorMap* tx = tensor_map(x.data_ptr(), M, K, K, ecz::gemm_block_n(M));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int rc = ecz::launch_gemm_cluster(tw, tx, nullptr, M, N, K, splits, status_word(x.device()), stream, &peer);
  TORCH_CHECK(rc == 0, "linear_push: unsupported shape or launch failure");
}

// ---- sequence-parallel tensor parallelism (tp_sp.cu) ----------------------------------------------------------
// A rank's buffer layout from (world, rank, hidden, max_rows, n_cap); returns its size in bytes.
int64_t sp_buffer_bytes(int64_t world, int64_t rank, int64_t hidden, int64_t max_rows, int64_t n_cap) {
  return ecz::sp_layout(world, rank, hidden, max_rows, n_cap).bytes;
}

ecz::SpLayout sp_check(const std::vector<int64_t>& ptrs, int64_t rank, int64_t hidden, int64_t max_rows,
                       int64_t n_cap) {
  TORCH_CHECK(!ptrs.empty() && rank >= 0 && rank < static_cast<int64_t>(ptrs.size()), "sp: bad rank or peers");
  return ecz::sp_layout(static_cast<int>(ptrs.size()), static_cast<int>(rank), static_cast<int>(hidden),
                        static_cast<int>(max_rows), static_cast<int>(n_cap));
}

// Reduce this rank's reduce-scatter partials (or, with partials = false, take resid alone), add the residual rows
// [rows, H], RMSNorm with w and all-gather the normed rows at row0; returns the new residual rows.
Tensor sp_reduce_norm(std::vector<int64_t> ptrs, int64_t rank, int64_t hidden, int64_t max_rows, int64_t n_cap,
                      bool partials, Tensor resid, Tensor w, double eps, int64_t row0, int64_t cap_slot) {
  CHECK_CUDA(w);
  CHECK_BF16(w);
  CHECK_BF16(resid);
  const ecz::SpLayout L = sp_check(ptrs, rank, hidden, max_rows, n_cap);
  c10::cuda::CUDAGuard guard(w.device());
  resid = resid.contiguous();
  TORCH_CHECK(resid.dim() == 2 && resid.size(1) == hidden && w.numel() == hidden, "sp_reduce_norm: resid [rows, H]");
  if (resid.numel() > 0) CHECK_ON(resid, w);
  auto out = at::empty_like(resid);
  const int rc = ecz::launch_sp_reduce_norm(peer_ptrs(ptrs), L, partials, resid.numel() ? resid.data_ptr() : nullptr,
                                            resid.numel() ? out.data_ptr() : nullptr, w.data_ptr(),
                                            static_cast<int>(resid.size(0)), static_cast<int>(row0),
                                            static_cast<float>(eps), static_cast<int>(cap_slot),
                                            status_word(w.device()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "sp_reduce_norm: rows, offset or capture slot outside the buffer");
  return out;
}

// Wait for the current all-gather round and return its rows [rows, H].
Tensor sp_fetch(std::vector<int64_t> ptrs, int64_t rank, int64_t hidden, int64_t max_rows, int64_t n_cap,
                int64_t rows, Tensor like) {
  const ecz::SpLayout L = sp_check(ptrs, rank, hidden, max_rows, n_cap);
  c10::cuda::CUDAGuard guard(like.device());
  auto out = at::empty({rows, hidden}, like.options().dtype(at::kBFloat16));
  const int rc = ecz::launch_sp_fetch(peer_ptrs(ptrs), L, out.data_ptr(), static_cast<int>(rows),
                                      status_word(like.device()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "sp_fetch: rows outside the buffer");
  return out;
}

// Captured residual rows [rows, H] of capture slot `slot` (valid once a later all-gather round was consumed).
Tensor sp_capture(std::vector<int64_t> ptrs, int64_t rank, int64_t hidden, int64_t max_rows, int64_t n_cap,
                  int64_t slot, int64_t rows, Tensor like) {
  const ecz::SpLayout L = sp_check(ptrs, rank, hidden, max_rows, n_cap);
  TORCH_CHECK(slot >= 0 && slot < n_cap && rows <= max_rows, "sp_capture: slot or rows outside the buffer");
  c10::cuda::CUDAGuard guard(like.device());
  auto out = at::empty({rows, hidden}, like.options().dtype(at::kBFloat16));
  const char* src = reinterpret_cast<const char*>(ptrs[rank]) + L.cap_off + slot * max_rows * hidden * 2;
  TORCH_CHECK(cudaMemcpyAsync(out.data_ptr(), src, rows * hidden * 2, cudaMemcpyDeviceToDevice,
                              at::cuda::getCurrentCUDAStream()) == cudaSuccess, "sp_capture: copy failed");
  return out;
}

// All-gather -> GEMM: y [rows, N] = X . w^T with X the current all-gather round's rows (the GEMM waits for them).
Tensor sp_linear_ag(std::vector<int64_t> ptrs, int64_t rank, int64_t hidden, int64_t max_rows, int64_t n_cap,
                    int64_t rows, Tensor w) {
  CHECK_CUDA(w);
  CHECK_BF16(w);
  const ecz::SpLayout L = sp_check(ptrs, rank, hidden, max_rows, n_cap);
  TORCH_CHECK(w.dim() == 2 && w.size(1) == hidden && rows >= 1 && rows <= max_rows, "sp_linear_ag: w [N, H]");
  c10::cuda::CUDAGuard guard(w.device());
  w = w.contiguous();
  const int M = static_cast<int>(rows), K = static_cast<int>(hidden), N = static_cast<int>(w.size(0));
  auto y = at::empty({M, N}, w.options());
  const char* ag = reinterpret_cast<const char*>(ptrs[rank]) + L.ag_off;
  const int bn = ecz::gemm_block_n(M);
  const CUtensorMap* tw = tensor_map(w.data_ptr(), N, K, K, 128);
  const CUtensorMap* tx0 = tensor_map(ag, M, K, K, bn);
  const CUtensorMap* tx1 = tensor_map(ag + static_cast<size_t>(max_rows) * hidden * 2, M, K, K, bn);
  ecz::AgWait wait;
  wait.ctrl = reinterpret_cast<unsigned*>(ptrs[rank]);
  wait.world = static_cast<int>(ptrs.size());
  const int sms = num_sms(w.get_device());
  const int rc = ecz::launch_gemm_cluster(tw, tx0, y.data_ptr(), M, N, K, ecz::gemm_cluster_splits(M, N, K, sms),
                                          status_word(w.device()), at::cuda::getCurrentCUDAStream(), nullptr, &wait,
                                          tx1);
  TORCH_CHECK(rc == 0, "sp_linear_ag: unsupported shape or launch failure");
  return y;
}

// All-gather -> GEMM on the swap-AB kernel for a consumer that fuses the split-K reduction (rope_store, the gated
// activation): the split-K partials [splits, rows, N] (fp32), or [rows, N] bf16 when K is not split, as linear_parts.
Tensor sp_linear_ag_parts(std::vector<int64_t> ptrs, int64_t rank, int64_t hidden, int64_t max_rows, int64_t n_cap,
                          int64_t rows, Tensor w) {
  CHECK_CUDA(w);
  CHECK_BF16(w);
  const ecz::SpLayout L = sp_check(ptrs, rank, hidden, max_rows, n_cap);
  TORCH_CHECK(w.dim() == 2 && w.size(1) == hidden && rows >= 1 && rows <= max_rows, "sp_linear_ag_parts: w [N, H]");
  const int M = static_cast<int>(rows), K = static_cast<int>(hidden), N = static_cast<int>(w.size(0));
  const int bn = ecz::gemm_block_n(M);
  TORCH_CHECK(bn <= 64, "sp_linear_ag_parts serves passes of at most 64 rows");
  c10::cuda::CUDAGuard guard(w.device());
  w = w.contiguous();
  const int sms = num_sms(w.get_device());
  int splits = std::min(8, ecz::gemm_splits(M, N, K, 2 * sms));
  const int total_kb = (K + 63) / 64, kbps = (total_kb + splits - 1) / splits;
  splits = (total_kb + kbps - 1) / kbps;  // the launcher drops empty splits the same way
  const char* ag = reinterpret_cast<const char*>(ptrs[rank]) + L.ag_off;
  const CUtensorMap* tw = tensor_map(w.data_ptr(), N, K, K, 128);
  const CUtensorMap* tx0 = tensor_map(ag, M, K, K, bn);
  const CUtensorMap* tx1 = tensor_map(ag + static_cast<size_t>(max_rows) * hidden * 2, M, K, K, bn);
  ecz::AgWait wait;
  wait.ctrl = reinterpret_cast<unsigned*>(ptrs[rank]);
  wait.world = static_cast<int>(ptrs.size());
  Tensor out = splits > 1 ? at::empty({splits, M, N}, w.options().dtype(at::kFloat)) : at::empty({M, N}, w.options());
  const int rc = ecz::launch_gemm_bf16(tw, tx0, splits > 1 ? nullptr : out.data_ptr(),
                                       splits > 1 ? out.data_ptr<float>() : nullptr, M, N, K, splits,
                                       status_word(w.device()), at::cuda::getCurrentCUDAStream(), nullptr, nullptr,
                                       3, &wait, tx1);
  TORCH_CHECK(rc == 0, "sp_linear_ag_parts: launch failed (", rc, ")");
  return out;
}

// GEMM -> reduce-scatter: x [rows, K] . w^T with every output row stored into its owner rank's partial slot.
void sp_linear_rs(std::vector<int64_t> ptrs, int64_t rank, int64_t hidden, int64_t max_rows, int64_t n_cap,
                  Tensor x, Tensor w) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  const ecz::SpLayout L = sp_check(ptrs, rank, hidden, max_rows, n_cap);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1) && w.size(0) == hidden,
              "sp_linear_rs expects x [M, K] and w [H, K]");
  TORCH_CHECK(x.size(0) >= 1 && x.size(0) <= max_rows, "sp_linear_rs: more rows than the buffer holds");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  w = w.contiguous();
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(hidden);
  ecz::PeerOut peer{};
  peer.ptrs = peer_ptrs(ptrs);
  peer.world = L.world;
  peer.rank = L.rank;
  peer.mode = 1;
  peer.shard_rows = (M + L.world - 1) / L.world;
  peer.shard_max = L.shard_max;
  peer.data_off = L.rs_off;
  const CUtensorMap* tw = tensor_map(w.data_ptr(), N, K, K, 128);
  const CUtensorMap* tx = tensor_map(x.data_ptr(), M, K, K, ecz::gemm_block_n(M));
  const int sms = num_sms(x.get_device());
  const int rc = ecz::launch_gemm_cluster(tw, tx, nullptr, M, N, K, ecz::gemm_cluster_splits(M, N, K, sms),
                                          status_word(x.device()), at::cuda::getCurrentCUDAStream(), &peer);
  TORCH_CHECK(rc == 0, "sp_linear_rs: unsupported shape or launch failure");
}

void push(Tensor src, std::vector<int64_t> ptrs, int64_t rank, int64_t parity, int64_t slot_elems) {
  CHECK_CUDA(src);
  CHECK_BF16(src);
  c10::cuda::CUDAGuard guard(src.device());
  src = src.contiguous();
  const int rc = ecz::launch_push(src.data_ptr(), src.numel(), peer_ptrs(ptrs), static_cast<int>(rank),
                                  static_cast<int>(ptrs.size()), static_cast<int>(parity), slot_elems,
                                  num_sms(src.get_device()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "push: size must be a multiple of 8 and fit the slot");
}

std::tuple<Tensor, Tensor> reduce_rmsnorm(std::vector<int64_t> ptrs, int64_t rank, int64_t parity, int64_t slot_elems,
                                          c10::optional<Tensor> resid, Tensor w, double eps, int64_t rows,
                                          int64_t hidden, Tensor like) {
  CHECK_CUDA(w);
  c10::cuda::CUDAGuard guard(w.device());
  auto out = at::empty({rows, hidden}, like.options());
  auto resid_out = at::empty({rows, hidden}, like.options());
  Tensor r;
  if (resid.has_value()) r = resid->contiguous();
  const int rc = ecz::launch_reduce_rmsnorm(peer_ptrs(ptrs), static_cast<int>(rank), static_cast<int>(ptrs.size()),
                                            static_cast<int>(parity), slot_elems,
                                            resid.has_value() ? r.data_ptr() : nullptr, w.data_ptr(), out.data_ptr(),
                                            resid_out.data_ptr(), static_cast<int>(rows), static_cast<int>(hidden),
                                            static_cast<float>(eps), status_word(w.device()),
                                            at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "reduce_rmsnorm: rows x hidden must fit the slot, hidden a multiple of 8");
  return {out, resid_out};
}

int64_t status(int64_t device) {
  const at::Device dev(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  c10::cuda::CUDAGuard guard(dev);
  unsigned* word = status_word(dev);
  unsigned host = 0;
  cudaMemcpy(&host, word, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (host != 0) cudaMemset(word, 0, sizeof(unsigned));
  return static_cast<int64_t>(host);
}

// Failure-detection probe: the expert-parallel segments kernel of a one-rank buffer waits for a dispatch that nothing
// sends; its bounded wait gives up after the device wait limit, sets the wait-peer status bit and returns. Returns the
// status word (cleared unless keep_status).
int64_t ep_wait_probe(int64_t ptr, int64_t experts_local, int64_t cap, int64_t hidden, int64_t ret_rows,
                      bool keep_status) {
  int device = 0;
  cudaGetDevice(&device);
  const at::Device dev(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  const ecz::EpLayout L = ecz::ep_layout(1, static_cast<int>(experts_local), static_cast<int>(cap),
                                         static_cast<int>(hidden), static_cast<int>(ret_rows));
  ecz::PeerPtrs peers{};
  peers.ptr[0] = reinterpret_cast<void*>(ptr);
  auto seg = at::empty({3, experts_local}, at::TensorOptions().dtype(at::kInt).device(dev));
  int* s0 = seg.data_ptr<int>();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(ecz::launch_ep_segments(peers, L, 0, s0, s0 + experts_local, s0 + 2 * experts_local, status_word(dev),
                                      stream) == 0, "ep_wait_probe: launch failed");
  cudaStreamSynchronize(stream);
  unsigned host = 0;
  cudaMemcpy(&host, status_word(dev), sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (!keep_status && host != 0) cudaMemset(status_word(dev), 0, sizeof(unsigned));
  return static_cast<int64_t>(host);
}

std::tuple<int64_t, int64_t, int64_t> attention_plan(int64_t B, int64_t T, int64_t H, int64_t Hkv, int64_t S,
                                                     int64_t sms, int64_t window) {
  const ecz::AttnPlan p = ecz::attention_plan(B, T, H, Hkv, S, sms, false, 128, static_cast<int>(window));
  return {p.m_tiles, p.splits, p.chunks_per_split};
}

int64_t gemm_splits(int64_t M, int64_t N, int64_t K, int64_t sms) { return ecz::gemm_splits(M, N, K, sms); }
int64_t gemm_cluster_splits(int64_t M, int64_t N, int64_t K, int64_t sms) {
  return ecz::gemm_cluster_splits(M, N, K, sms);
}

}  // namespace

// Raises a formatted error: a host-only check that exceptions thrown in this library reach Python.
void raise_formatted(int64_t n) { TORCH_CHECK(n < 0, "formatted error ", n, " from economize_b200._C"); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "economize_b200 sm_100a kernels (tcgen05 / TMA)";
  m.def("rmsnorm", &rmsnorm, "fused residual add + RMSNorm");
  m.def("rope_store", &rope_store, "rotary embedding + KV-cache write (+ optional QK-norm; fp8 caches quantize)",
        py::arg("qkv"), py::arg("positions"), py::arg("cos"), py::arg("sin"), py::arg("H"), py::arg("Hkv"),
        py::arg("D"), py::arg("k_cache"), py::arg("v_cache"), py::arg("kv_len"), py::arg("n_new"), py::arg("q_norm"),
        py::arg("k_norm"), py::arg("eps"), py::arg("q_offset"), py::arg("k_scale") = py::none(),
        py::arg("v_scale") = py::none(), py::arg("pages") = py::none());
  m.def("attention", &attention, "tree-masked / causal attention over the slot cache (tcgen05; bf16 or fp8 KV)",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("kv_len"), py::arg("n_new"), py::arg("mask"),
        py::arg("scale"), py::arg("q_offset"), py::arg("trace") = py::none(), py::arg("k_scale") = py::none(),
        py::arg("v_scale") = py::none(), py::arg("keep") = py::none(), py::arg("lse_out") = py::none(),
        py::arg("kivi") = py::none(), py::arg("kivi_chunks") = py::none(), py::arg("kivi_bits") = 0,
        py::arg("tail") = 0, py::arg("softcap") = 0.0, py::arg("sinks") = py::none(), py::arg("window") = 0,
        py::arg("pages") = py::none());
  m.def("kivi_chunk_size", &ecz::kivi_chunk_size, "bytes of one KIVI-coded 128-key chunk");
  m.def("kivi_quantize", &kivi_quantize, "quantise committed cache chunks to KIVI codes and advance the counts",
        py::arg("cache"), py::arg("kivi"), py::arg("kv_len"), py::arg("chunks"), py::arg("bits"), py::arg("residual"),
        py::arg("max_new"), py::arg("pages") = py::none());
  m.def("attention_scores", &attention_scores, "accumulate KV-eviction attention scores (tcgen05)", py::arg("q"),
        py::arg("k_cache"), py::arg("kv_len"), py::arg("n_new"), py::arg("mask"), py::arg("lse2"), py::arg("scores"),
        py::arg("scale"), py::arg("q_offset"), py::arg("pages") = py::none());
  m.def("silu_mul", &silu_mul, "SwiGLU activation of [gate; up]");
  m.def("vs_keep", &vs_keep, "MInference vertical-slash pattern -> per-KV-head keep bit words");
  m.def("hadamard", &hadamard, "block Walsh-Hadamard transform of the last dimension (QuaRot online rotation)");
  m.def("glu_hadamard", &glu_hadamard, "act(gate) * up of [gate; up] followed by the block Hadamard transform");
  m.def("glu", &glu_act, "act(gate) * up of [gate; up]: act 0 = SiLU, 1 = GELU (tanh approximation), 2 = clamped "
        "SwiGLU with the given limit", py::arg("gu"), py::arg("act"), py::arg("limit") = 7.0);
  m.def("linear_parts", &linear_parts, "x @ w.T as bf16 or fp32 split-K partials for a fusing consumer");
  m.def("moe_route", &moe_route, "top-k expert routing with deterministic expert-order positions");
  m.def("moe_gather", &moe_gather, "permute token rows into expert order");
  m.def("moe_combine", &moe_combine, "weighted sum of each token's expert outputs");
  m.def("linear_grouped", &linear_grouped, "grouped expert GEMM over expert-ordered rows (tcgen05)");
  m.def("linear_fp8", &linear_fp8, "block-scaled fp8 linear (1x128 activation / 128x128 weight scales)",
        py::arg("x"), py::arg("wq"), py::arg("sw"), py::arg("splits") = 0);
  m.def("topk_logp", &topk_logp, "fused log-softmax + top-k (+ draft-to-target id map)", py::arg("logits"),
        py::arg("k"), py::arg("floor"), py::arg("d2t") = py::none());
  m.def("linear_sp24", &linear_sp24, "2:4 sparse linear (kept values + positions, expanded in shared memory)",
        py::arg("x"), py::arg("values"), py::arg("meta"), py::arg("splits") = 0);
  m.def("linear_variant", &linear_variant, "x @ w.T through an explicit GEMM variant (tuning)");
  m.def("gemm_cluster_capacity", &gemm_cluster_capacity, "resident clusters of the split-K cluster GEMM");
  m.def("raise_formatted", &raise_formatted, "raise a formatted RuntimeError (exception-path self test)");
  m.def("linear", &linear_bf16, "x @ w.T on tcgen05 (swap-AB, split-K)");
  m.def("linear_wq", &linear_wq, "weight-only quantized x @ dequant(w).T (int4 / int8 / fp8 weights)", py::arg("x"),
        py::arg("qweight"), py::arg("scales"), py::arg("zeros"), py::arg("fmt"), py::arg("group"), py::arg("splits") = 0);
  m.def("argmax", &argmax, "row argmax");
  m.def("greedy_accept", &greedy_accept, "longest accepted path of a verified draft tree", py::arg("tokens"),
        py::arg("parents"), py::arg("pred"), py::arg("ok") = py::none());
  m.def("kv_compact", &kv_compact, "move an accepted path's K/V to consecutive slots", py::arg("cache"),
        py::arg("kv_len"), py::arg("path"), py::arg("n_acc"), py::arg("pages") = py::none());
  m.def("sample", &sample, "inverse-CDF draw of one token per probability row");
  m.def("rejection", &rejection, "lossless speculative sampling of a draft chain (accept/reject + resample)");
  m.def("ngram", &ngram, "prompt-lookup draft proposals from the token history");
  m.def("tree_expand", &tree_expand, "one depth of dynamic-tree drafting bookkeeping (in place)");
  m.def("tree_layout", &tree_layout, "ancestor bits and positions of a verified tree", py::arg("parents"),
        py::arg("kv_len"));
  m.def("tree_select", &tree_select, "the best candidates of a draft tree in candidate order, parents remapped");
  m.def("sign_matvec", &sign_matvec, "x times a packed sign matrix (LittleBit factors, <= 16 rows)");
  m.def("colsparse_linear", &colsparse_linear, "activation-sparse GEMV over a transposed weight (<= 16 rows)");
  m.def("glu_rows", &glu_rows, "gated-MLP hidden over the kept channels only (CATS / Deja Vu, <= 16 rows)");
  m.def("ep_buffer_bytes", &ep_buffer_bytes, "bytes of one rank's expert-parallel symmetric buffer");
  m.def("ep_wait_probe", &ep_wait_probe, "run one bounded device wait that nothing satisfies; return the status",
        py::arg("ptr"), py::arg("experts_local"), py::arg("cap"), py::arg("hidden"), py::arg("ret_rows"),
        py::arg("keep_status") = false);
  m.def("ep_moe", &ep_moe, "expert-parallel MoE MLP with NVLink peer-store dispatch and combine");
  m.def("symm_alloc", &symm_alloc, "cudaMalloc an IPC-exportable buffer: (pointer, handle)");
  m.def("symm_open", &symm_open, "map a peer's buffer from its IPC handle");
  m.def("symm_close", &symm_close, "unmap a peer's buffer");
  m.def("symm_free", &symm_free, "free an own symmetric buffer");
  m.def("symm_control_bytes", &symm_control_bytes, "bytes of the control block before the data slots");
  m.def("push", &push, "store this rank's partial into every peer's slot and signal arrival");
  m.def("linear_push", &linear_push, "row-parallel GEMM whose output tiles go into every peer's slot");
  m.def("sp_buffer_bytes", &sp_buffer_bytes, "bytes of one rank's sequence-parallel buffer");
  m.def("sp_reduce_norm", &sp_reduce_norm, "reduce-scatter partials + residual + RMSNorm, all-gather the rows");
  m.def("sp_fetch", &sp_fetch, "wait for the current all-gather round and copy its rows");
  m.def("sp_capture", &sp_capture, "copy the captured residual rows of a capture slot");
  m.def("sp_linear_ag_parts", &sp_linear_ag_parts, "all-gather -> split-K GEMM whose partials a fused consumer sums");
  m.def("sp_linear_ag", &sp_linear_ag, "all-gather -> GEMM (the GEMM waits for every rank's rows)");
  m.def("sp_linear_rs", &sp_linear_rs, "GEMM -> reduce-scatter (rows stored into their owner's partial slot)");
  m.def("reduce_rmsnorm", &reduce_rmsnorm, "wait for every rank's partial, sum, add residual, RMSNorm");
  m.def("status", &status, "read and clear the device status word of bounded waits");
  m.def("attention_plan", &attention_plan, "(m_tiles, splits, chunks_per_split) of an attention launch",
        py::arg("B"), py::arg("T"), py::arg("H"), py::arg("Hkv"), py::arg("S"), py::arg("sms"), py::arg("window") = 0);
  m.def("gemm_splits", &gemm_splits, "split-K factor of a GEMM launch");
  m.def("gemm_cluster_splits", &gemm_cluster_splits, "cluster size of the cluster split-K GEMM");
}
