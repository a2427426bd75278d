// PyTorch operator layer of the B200 fused sampler: module `fused_sampling`.
//
// Same names, arguments, return types and error messages as the reference extension
// (csrc/bindings.cpp:16-25, csrc/fused_sampling.cu:337-540). The only work done here is
// unpacking tensors, the current stream and torch's generator state; every computation goes
// through the C ABI of libfs_b200.so (include/fused_sampling_b200.h).
#include <ATen/core/CachingHostAllocator.h>
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAGeneratorImpl.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <optional>
#include <string>
#include <tuple>
#include <vector>

#include "fused_sampling_b200.h"

namespace {

// Where a call's logits live. A cuda tensor runs on its own device. A tensor in pinned host
// memory (deliberate extension of the reference, which takes cuda tensors only) is read in place
// by the kernels over PCIe -- pinned pages are mapped into every device's address space -- on the
// current CUDA device, with no copy-engine transfer; the call's outputs are then pinned host
// tensors that the kernels write directly. Like a non_blocking copy to the host, they hold their
// values once the stream has reached the call.
struct Source {
  const void* ptr = nullptr;  // device-accessible address of the logits
  bool host = false;          // pinned host memory
  c10::Device device = c10::Device(c10::kCUDA, 0);
  torch::TensorOptions opts;  // outputs: on the logits' device, or in pinned host memory
};

// Deliberate difference to the reference: top_k may be anything up to the vocabulary size
// (the reference rejected top_k > 128, csrc/fused_sampling.cu:351).
Source check_logits(const torch::Tensor& logits, bool allow_host = false) {
  // one driver query tells pinned (and mapped) host memory apart from pageable memory
  cudaPointerAttributes at = {};
  bool host = false;
  if (allow_host && !logits.is_cuda() && logits.device().is_cpu()) {
    const cudaError_t e = cudaPointerGetAttributes(&at, logits.data_ptr());
    if (e != cudaSuccess) cudaGetLastError();
    host = e == cudaSuccess && at.type == cudaMemoryTypeHost;
  }
  TORCH_CHECK((logits.is_cuda() || host) && logits.dim() == 2 && logits.stride(1) == 1 &&
                  logits.stride(0) >= logits.size(1),
              allow_host ? "logits must be a contiguous cuda [B, V] tensor (or one in pinned host memory)"
                         : "logits must be a contiguous cuda [B, V] tensor");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kHalf,
              "logits must be float16 or bfloat16");
  TORCH_CHECK(logits.size(0) >= 1 && logits.size(1) >= 1, "logits must be a non-empty [B, V] tensor");
  Source src;
  if (!host) {
    src.ptr = logits.data_ptr();
    src.device = logits.device();
    src.opts = logits.options();
    return src;
  }
  TORCH_CHECK(at.devicePointer != nullptr, "pinned host logits are not mapped into the device address space");
  src.ptr = at.devicePointer;
  src.host = true;
  src.device = c10::Device(c10::kCUDA, c10::cuda::current_device());
  src.opts = logits.options().pinned_memory(true);
  return src;
}

// Host tensors that the call's kernels read or write stay out of the pinned-memory cache's reuse
// until the stream has passed the call (what torch does for a non_blocking host copy).
void hold_host(const Source& src, std::initializer_list<const torch::Tensor*> ts) {
  if (!src.host) return;
  const c10::Stream stream = at::cuda::getCurrentCUDAStream().unwrap();
  for (const torch::Tensor* t : ts) {
    if (t == nullptr || !t->defined()) continue;
    const auto& dp = t->storage().data_ptr();
    at::getHostAllocator(at::kCUDA)->record_event(dp.get(), dp.get_context(), stream);
  }
}

void check_top_k(int64_t top_k) { TORCH_CHECK(top_k >= 1, "top_k must be >= 1"); }

void check_top_p(double top_p) {
  TORCH_CHECK(top_p > 0.0 && top_p <= 1.0, "top_p must be in (0, 1]");
}

void check(fs_status st, const char* what) {
  TORCH_CHECK(st == FS_OK, what, " failed (status ", static_cast<int>(st), "): ", fs_last_error());
}

fs_stream_t current_stream() {
  return reinterpret_cast<fs_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

// Reference top_p is a double compared as p >= 1.0 before narrowing (benchmarks/reference.py:58).
float narrow_top_p(double top_p) { return top_p >= 1.0 ? 1.0f : static_cast<float>(top_p); }

fs_sample_args base_args(const torch::Tensor& logits, const Source& src, int64_t top_k, double top_p,
                         int64_t splits) {
  fs_sample_args a = {};
  a.logits = src.ptr;
  // pinned host logits were written by the CPU before this call: no kernel still running writes them
  if (src.host) a.input_flags = FS_INPUT_READY;
  a.dtype = logits.scalar_type() == at::kBFloat16 ? FS_BF16 : FS_F16;
  a.batch = logits.size(0);
  a.vocab = logits.size(1);
  a.row_stride = logits.stride(0);
  a.id_base = 0;
  a.top_k = top_k;
  a.top_p = narrow_top_p(top_p);
  a.splits = static_cast<int32_t>(splits);
  return a;
}

// (seed, offset) by value, or torch's default CUDA generator when offset < 0 (graph-safe:
// under capture the kernel reads seed/offset through pointers, like at::cuda::philox::unpack).
void set_rng(fs_rng* rng, int64_t seed, int64_t offset) {
  if (offset >= 0) {
    rng->seed = static_cast<uint64_t>(seed);
    rng->offset = static_cast<uint64_t>(offset);
    return;
  }
  auto gen = at::get_generator_or_default<at::CUDAGeneratorImpl>(
      std::nullopt, at::cuda::detail::getDefaultCUDAGenerator());
  std::lock_guard<std::mutex> lock(gen->mutex_);
  const at::PhiloxCudaState st = gen->philox_cuda_state(4);
  if (st.captured_) {
    rng->seed_ptr = st.seed_.ptr;
    rng->offset_ptr = st.offset_.ptr;
    rng->offset_intragraph = st.offset_intragraph_;
  } else {
    rng->seed = st.seed_.val;
    rng->offset = st.offset_.val;
  }
}

int64_t clamp_k(const torch::Tensor& logits, int64_t top_k) { return std::min(top_k, logits.size(1)); }

// Device workspace for the streaming path, from torch's caching allocator (stream-ordered, so it
// may be released as soon as the launches are enqueued). Empty when the plan needs none.
torch::Tensor attach_workspace(fs_sample_args* a, c10::Device device) {
  const uint64_t bytes = fs_workspace_size(a);
  if (bytes == 0) return torch::Tensor();
  auto ws = torch::empty({static_cast<int64_t>(bytes)}, torch::TensorOptions().device(device).dtype(torch::kUInt8));
  a->workspace = ws.data_ptr();
  a->workspace_bytes = bytes;
  return ws;
}

torch::Tensor empty_i64(const torch::Tensor& like, at::IntArrayRef shape) {
  return torch::empty(shape, like.options().dtype(torch::kInt64));
}

torch::Tensor empty_out(const Source& src, at::IntArrayRef shape, at::ScalarType dt) {
  return torch::empty(shape, src.opts.dtype(dt));
}

}  // namespace

torch::Tensor sample_fused(torch::Tensor logits, int64_t top_k, double top_p, int64_t seed,
                           int64_t offset, int64_t splits_override) {
  check_top_p(top_p);
  const Source src = check_logits(logits, true);
  check_top_k(top_k);
  c10::cuda::CUDAGuard guard(src.device);
  auto out = empty_out(src, {logits.size(0)}, torch::kInt64);
  fs_sample_args a = base_args(logits, src, top_k, top_p, splits_override);
  set_rng(&a.rng, seed, offset);
  a.out_ids = out.data_ptr<int64_t>();
  auto ws = attach_workspace(&a, src.device);
  check(fs_sample(&a, current_stream()), "fs_sample");
  hold_host(src, {&logits, &out});
  return out;
}

torch::Tensor topk_fused(torch::Tensor logits, int64_t top_k, int64_t splits_override) {
  const Source src = check_logits(logits, true);
  check_top_k(top_k);
  c10::cuda::CUDAGuard guard(src.device);
  const int64_t K = clamp_k(logits, top_k);
  auto ids = empty_out(src, {logits.size(0), K}, torch::kInt64);
  fs_sample_args a = base_args(logits, src, top_k, 1.0, splits_override);
  a.topk_ids = ids.data_ptr<int64_t>();
  auto ws = attach_workspace(&a, src.device);
  check(fs_topk(&a, current_stream()), "fs_topk");
  hold_host(src, {&logits, &ids});
  return ids;
}

std::vector<torch::Tensor> stages_fused(torch::Tensor logits, int64_t top_k, double top_p,
                                        int64_t seed, int64_t offset, int64_t splits_override) {
  check_top_p(top_p);
  const Source src = check_logits(logits, true);
  check_top_k(top_k);
  c10::cuda::CUDAGuard guard(src.device);
  const int64_t B = logits.size(0), K = clamp_k(logits, top_k);
  auto out = empty_out(src, {B}, torch::kInt64);
  auto keep = empty_out(src, {B, K}, torch::kBool);
  auto renormed = empty_out(src, {B, K}, torch::kFloat32);
  fs_sample_args a = base_args(logits, src, top_k, top_p, splits_override);
  a.rng.seed = static_cast<uint64_t>(seed);
  a.rng.offset = static_cast<uint64_t>(offset);
  a.out_ids = out.data_ptr<int64_t>();
  a.keep = reinterpret_cast<uint8_t*>(keep.data_ptr<bool>());
  a.renormed = renormed.data_ptr<float>();
  auto ws = attach_workspace(&a, src.device);
  check(fs_sample(&a, current_stream()), "fs_sample");
  hold_host(src, {&logits, &out, &keep, &renormed});
  return {out, keep, renormed};
}

torch::Tensor probe_phase(torch::Tensor logits, int64_t top_k, double top_p, int64_t phase,
                          int64_t splits_override) {
  TORCH_CHECK(phase >= 1 && phase <= FS_NUM_PHASES, "phase must be in [1, ", FS_NUM_PHASES, "]");
  check_top_p(top_p);
  const Source src = check_logits(logits);
  check_top_k(top_k);
  c10::cuda::CUDAGuard guard(logits.device());
  auto out = empty_i64(logits, {logits.size(0)});
  fs_sample_args a = base_args(logits, src, top_k, top_p, splits_override);
  a.out_ids = out.data_ptr<int64_t>();
  a.stop_phase = static_cast<int32_t>(phase);
  check(fs_probe_phase(&a, current_stream()), "fs_probe_phase");
  return out;
}

using AttrRow = std::tuple<std::string, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t>;

std::vector<AttrRow> kernel_attrs() {
  const int32_t n = fs_kernel_attrs(nullptr, 0);
  TORCH_CHECK(n >= 0, "fs_kernel_attrs failed: ", fs_last_error());
  std::vector<fs_kernel_attr> rows(static_cast<size_t>(n));
  fs_kernel_attrs(rows.data(), n);
  std::vector<AttrRow> out;
  for (const auto& r : rows)
    out.emplace_back(r.name, r.param, r.block, r.regs, r.local_bytes, r.static_smem, r.blocks_per_sm);
  return out;
}

torch::Tensor probe_noop(torch::Tensor logits) {
  check_logits(logits);
  c10::cuda::CUDAGuard guard(logits.device());
  auto out = empty_i64(logits, {logits.size(0)});
  check(fs_probe_noop(out.data_ptr<int64_t>(), logits.size(0), current_stream()), "fs_probe_noop");
  return out;
}

torch::Tensor probe_scan_rowblock(torch::Tensor logits) {
  check_logits(logits);
  c10::cuda::CUDAGuard guard(logits.device());
  auto out = empty_i64(logits, {logits.size(0)});
  const int32_t dt = logits.scalar_type() == at::kBFloat16 ? FS_BF16 : FS_F16;
  check(fs_probe_scan_rowblock(logits.data_ptr(), dt, logits.size(0), logits.size(1),
                               logits.stride(0), out.data_ptr<int64_t>(), current_stream()),
        "fs_probe_scan_rowblock");
  return out;
}

torch::Tensor probe_scan_split(torch::Tensor logits, int64_t splits) {
  check_logits(logits);
  TORCH_CHECK(splits >= 1, "splits must be >= 1");
  c10::cuda::CUDAGuard guard(logits.device());
  auto out = empty_i64(logits, {logits.size(0)});
  const int32_t dt = logits.scalar_type() == at::kBFloat16 ? FS_BF16 : FS_F16;
  check(fs_probe_scan_split(logits.data_ptr(), dt, logits.size(0), logits.size(1), logits.stride(0),
                            static_cast<int32_t>(std::min<int64_t>(splits, 16)),
                            out.data_ptr<int64_t>(), current_stream()),
        "fs_probe_scan_split");
  return out;
}

// ---- extensions beyond the reference surface ----------------------------------------------

namespace {

void fill_rows(fs_sample_args* a, c10::Device device,
               const std::optional<torch::Tensor>& top_k_rows,
               const std::optional<torch::Tensor>& top_p_rows,
               const std::optional<torch::Tensor>& uniforms, int64_t B) {
  if (top_k_rows.has_value()) {
    const auto& t = *top_k_rows;
    TORCH_CHECK(t.is_cuda() && t.device() == device && t.scalar_type() == at::kInt &&
                    t.dim() == 1 && t.size(0) == B && t.is_contiguous(),
                "top_k_rows must be a contiguous int32 [B] tensor on the device the call runs on");
    a->top_k_rows = t.data_ptr<int32_t>();
  }
  if (top_p_rows.has_value()) {
    const auto& t = *top_p_rows;
    TORCH_CHECK(t.is_cuda() && t.device() == device && t.scalar_type() == at::kFloat &&
                    t.dim() == 1 && t.size(0) == B && t.is_contiguous(),
                "top_p_rows must be a contiguous float32 [B] tensor on the device the call runs on");
    a->top_p_rows = t.data_ptr<float>();
  }
  if (uniforms.has_value()) {
    const auto& t = *uniforms;
    TORCH_CHECK(t.is_cuda() && t.device() == device && t.scalar_type() == at::kFloat &&
                    t.dim() == 1 && t.size(0) == B && t.is_contiguous(),
                "uniforms must be a contiguous float32 [B] tensor on the device the call runs on");
    a->rng.uniforms = t.data_ptr<float>();
  }
}

}  // namespace

// General form: per-row k / p tensors, caller-supplied uniforms, vocab-shard id base, RNG row
// base, optional stage outputs and per-row status. Returns
// (ids[B], topk_ids[B,K] | None, keep[B,K] | None, renormed[B,K] | None, status[B]).
std::vector<std::optional<torch::Tensor>> sample_ex(
    torch::Tensor logits, int64_t top_k, double top_p, std::optional<torch::Tensor> top_k_rows,
    std::optional<torch::Tensor> top_p_rows, std::optional<torch::Tensor> uniforms, int64_t seed,
    int64_t offset, int64_t splits, int64_t id_base, int64_t row_base, bool return_stages, int64_t path,
    double temperature) {
  const Source src = check_logits(logits, true);
  check_top_k(top_k);
  if (!top_p_rows.has_value()) check_top_p(top_p);
  c10::cuda::CUDAGuard guard(src.device);
  const int64_t B = logits.size(0), K = clamp_k(logits, top_k);
  auto out = empty_out(src, {B}, torch::kInt64);
  auto status = empty_out(src, {B}, torch::kInt32);
  fs_sample_args a = base_args(logits, src, top_k, top_p_rows.has_value() ? 1.0 : top_p, splits);
  a.id_base = id_base;
  fill_rows(&a, src.device, top_k_rows, top_p_rows, uniforms, B);
  if (!uniforms.has_value()) set_rng(&a.rng, seed, offset);
  a.rng.row_base = row_base;
  a.out_ids = out.data_ptr<int64_t>();
  a.row_status = status.data_ptr<int32_t>();
  std::optional<torch::Tensor> ids, keep, ren;
  if (return_stages) {
    ids = empty_out(src, {B, K}, torch::kInt64);
    keep = empty_out(src, {B, K}, torch::kBool);
    ren = empty_out(src, {B, K}, torch::kFloat32);
    a.topk_ids = ids->data_ptr<int64_t>();
    a.keep = reinterpret_cast<uint8_t*>(keep->data_ptr<bool>());
    a.renormed = ren->data_ptr<float>();
  }
  a.path = static_cast<int32_t>(path);
  a.temperature = static_cast<float>(temperature);
  auto ws = attach_workspace(&a, src.device);
  check(fs_sample(&a, current_stream()), "fs_sample");
  hold_host(src, {&logits, &out, &status, ids ? &*ids : nullptr, keep ? &*keep : nullptr, ren ? &*ren : nullptr});
  return {out, ids, keep, ren, status};
}

// Vocab-shard local half: [B, K + 1] packed candidates (uint64 bit patterns in an int64 tensor).
// `out`, when given, is a contiguous int64 cuda [B, top_k + 1] tensor (e.g. one part of a
// [parts, B, top_k + 1] block) that receives the candidates.
torch::Tensor shard_candidates(torch::Tensor logits, int64_t top_k, int64_t id_base, int64_t splits,
                               std::optional<torch::Tensor> out) {
  const Source src = check_logits(logits);
  check_top_k(top_k);
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t B = logits.size(0);
  TORCH_CHECK(top_k <= logits.size(1), "shard top_k must not exceed the shard vocabulary");
  torch::Tensor cand;
  if (out.has_value()) {
    cand = *out;
    TORCH_CHECK(cand.is_cuda() && cand.device() == logits.device() && cand.scalar_type() == at::kLong &&
                    cand.dim() == 2 && cand.size(0) == B && cand.size(1) == top_k + 1 && cand.is_contiguous(),
                "out must be a contiguous int64 cuda [B, top_k + 1] tensor on the logits' device");
  } else {
    cand = empty_i64(logits, {B, top_k + 1});
  }
  fs_sample_args a = base_args(logits, src, top_k, 1.0, splits);
  a.id_base = id_base;
  auto ws = attach_workspace(&a, logits.device());
  check(fs_shard_candidates(&a, reinterpret_cast<uint64_t*>(cand.data_ptr<int64_t>()), current_stream()),
        "fs_shard_candidates");
  return cand;
}

// Vocab-shard merge half over gathered candidates [parts, B, K + 1]; `bf16` selects the logit
// format the keys encode. Returns (ids[B], status[B]).
std::vector<torch::Tensor> merge_sample(torch::Tensor cand, bool bf16, int64_t top_k, double top_p,
                                        std::optional<torch::Tensor> top_k_rows,
                                        std::optional<torch::Tensor> top_p_rows,
                                        std::optional<torch::Tensor> uniforms, int64_t seed,
                                        int64_t offset, int64_t row_base, double temperature) {
  TORCH_CHECK(cand.is_cuda() && cand.dim() == 3 && cand.is_contiguous() &&
                  cand.scalar_type() == at::kLong,
              "cand must be a contiguous int64 cuda [parts, B, K + 1] tensor");
  check_top_k(top_k);
  TORCH_CHECK(cand.size(2) == top_k + 1, "cand rows must hold top_k + 1 words");
  if (!top_p_rows.has_value()) check_top_p(top_p);
  c10::cuda::CUDAGuard guard(cand.device());
  const int64_t parts = cand.size(0), B = cand.size(1);
  auto out = empty_i64(cand, {B});
  auto status = torch::empty({B}, cand.options().dtype(torch::kInt32));
  fs_sample_args a = {};
  a.dtype = bf16 ? FS_BF16 : FS_F16;
  a.batch = B;
  a.top_k = top_k;
  a.top_p = top_p_rows.has_value() ? 1.0f : narrow_top_p(top_p);
  fill_rows(&a, cand.device(), top_k_rows, top_p_rows, uniforms, B);
  if (!uniforms.has_value()) set_rng(&a.rng, seed, offset);
  a.rng.row_base = row_base;
  a.out_ids = out.data_ptr<int64_t>();
  a.row_status = status.data_ptr<int32_t>();
  a.temperature = static_cast<float>(temperature);
  check(fs_merge_sample(&a, reinterpret_cast<const uint64_t*>(cand.data_ptr<int64_t>()),
                        static_cast<int32_t>(parts), current_stream()),
        "fs_merge_sample");
  return {out, status};
}

// Peer-to-peer exchange + merge (fs_tp_merge_sample): local_cand [B, K + 1] from
// shard_candidates; recv [2, world, max_batch, K + 1] int64 and flags [2, world, max_batch] int32
// on this rank's GPU; peer_recv / peer_flags: int64 cuda [world] tensors of device pointers;
// epoch_counter: optional int32 [2] on this GPU (zeroed once), which replaces `epoch`.
std::vector<torch::Tensor> tp_merge(torch::Tensor local_cand, bool bf16, int64_t top_k, double top_p,
                                    torch::Tensor recv, torch::Tensor flags, torch::Tensor peer_recv,
                                    torch::Tensor peer_flags, int64_t world, int64_t rank, int64_t epoch,
                                    std::optional<torch::Tensor> uniforms, int64_t seed, int64_t offset,
                                    int64_t row_base, int64_t wait_polls, double temperature,
                                    std::optional<torch::Tensor> epoch_counter) {
  TORCH_CHECK(local_cand.is_cuda() && local_cand.dim() == 2 && local_cand.is_contiguous() &&
                  local_cand.scalar_type() == at::kLong && local_cand.size(1) == top_k + 1,
              "local_cand must be a contiguous int64 cuda [B, top_k + 1] tensor");
  TORCH_CHECK(recv.is_cuda() && recv.dim() == 4 && recv.is_contiguous() && recv.scalar_type() == at::kLong &&
                  recv.size(0) == 2 && recv.size(1) == world && recv.size(3) == top_k + 1,
              "recv must be a contiguous int64 cuda [2, world, max_batch, top_k + 1] tensor");
  TORCH_CHECK(flags.is_cuda() && flags.dim() == 3 && flags.is_contiguous() && flags.scalar_type() == at::kInt &&
                  flags.size(0) == 2 && flags.size(1) == world && flags.size(2) == recv.size(2),
              "flags must be a contiguous int32 cuda [2, world, max_batch] tensor");
  TORCH_CHECK(peer_recv.is_cuda() && peer_recv.numel() == world && peer_recv.scalar_type() == at::kLong &&
                  peer_flags.is_cuda() && peer_flags.numel() == world && peer_flags.scalar_type() == at::kLong,
              "peer_recv / peer_flags must be int64 cuda [world] tensors of device pointers");
  check_top_k(top_k);
  check_top_p(top_p);
  c10::cuda::CUDAGuard guard(local_cand.device());
  const int64_t B = local_cand.size(0);
  auto out = empty_i64(local_cand, {B});
  auto status = torch::empty({B}, local_cand.options().dtype(torch::kInt32));
  fs_sample_args a = {};
  a.dtype = bf16 ? FS_BF16 : FS_F16;
  a.batch = B;
  a.top_k = top_k;
  a.top_p = narrow_top_p(top_p);
  fill_rows(&a, local_cand.device(), std::nullopt, std::nullopt, uniforms, B);
  if (!uniforms.has_value()) set_rng(&a.rng, seed, offset);
  a.rng.row_base = row_base;
  a.out_ids = out.data_ptr<int64_t>();
  a.row_status = status.data_ptr<int32_t>();
  a.temperature = static_cast<float>(temperature);
  fs_tp_peers tp = {};
  tp.world = static_cast<int32_t>(world);
  tp.rank = static_cast<int32_t>(rank);
  tp.max_batch = recv.size(2);
  tp.epoch = static_cast<uint32_t>(epoch);
  if (epoch_counter.has_value()) {
    const auto& c = *epoch_counter;
    TORCH_CHECK(c.is_cuda() && c.scalar_type() == at::kInt && c.numel() >= 2 && c.is_contiguous() &&
                    c.device() == local_cand.device(),
                "epoch_counter must be a contiguous int32 cuda tensor of 2 words on the candidates' device");
    tp.epoch_counter = reinterpret_cast<uint32_t*>(c.data_ptr<int32_t>());
  }
  tp.wait_polls = wait_polls;
  tp.recv = reinterpret_cast<uint64_t*>(recv.data_ptr<int64_t>());
  tp.flags = reinterpret_cast<uint32_t*>(flags.data_ptr<int32_t>());
  tp.peer_recv = reinterpret_cast<uint64_t* const*>(peer_recv.data_ptr<int64_t>());
  tp.peer_flags = reinterpret_cast<uint32_t* const*>(peer_flags.data_ptr<int64_t>());
  check(fs_tp_merge_sample(&a, reinterpret_cast<const uint64_t*>(local_cand.data_ptr<int64_t>()), &tp,
                           current_stream()),
        "fs_tp_merge_sample");
  return {out, status};
}

std::tuple<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t> plan(
    int64_t batch, int64_t vocab, int64_t top_k, int64_t splits) {
  fs_plan_info p = {};
  check(fs_plan(batch, vocab, top_k, static_cast<int32_t>(splits), &p), "fs_plan");
  return {p.splits, p.chunks, p.threads, p.capacity, p.maxima_per_thread, p.lanes_per_max, p.smem_bytes,
          p.path, static_cast<int64_t>(p.workspace_bytes)};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("probe_noop", &probe_noop, "launch floor: allocate [B] and write it");
  m.def("probe_scan_rowblock", &probe_scan_rowblock, "one full pass, one block per row");
  m.def("probe_scan_split", &probe_scan_split, "one full pass, row split over a cluster");
  m.def("sample_fused", &sample_fused, "fused top-k + top-p + sample, [B, V] -> [B]");
  m.def("topk_fused", &topk_fused, "debug: the selected candidate ids, descending");
  m.def("stages_fused", &stages_fused, "debug: (token_ids, keep, renormed)");
  m.def("probe_phase", &probe_phase, "ablation: run phases 1..n of the pipeline and stop");
  m.def("kernel_attrs", &kernel_attrs, "debug: registers, spills, smem, occupancy per kernel");
  m.def("sample_ex", &sample_ex, "general sampler: per-row k/p, uniforms, id/row base, stages",
        py::arg("logits"), py::arg("top_k"), py::arg("top_p"), py::arg("top_k_rows") = py::none(),
        py::arg("top_p_rows") = py::none(), py::arg("uniforms") = py::none(), py::arg("seed") = 0,
        py::arg("offset") = -1, py::arg("splits") = 0, py::arg("id_base") = 0,
        py::arg("row_base") = 0, py::arg("return_stages") = false, py::arg("path") = 0,
        py::arg("temperature") = 1.0);
  m.def("shard_candidates", &shard_candidates, "vocab-shard local top-k as packed candidates",
        py::arg("logits"), py::arg("top_k"), py::arg("id_base"), py::arg("splits") = 0,
        py::arg("out") = py::none());
  m.def("merge_sample", &merge_sample, "merge gathered shard candidates and sample",
        py::arg("cand"), py::arg("bf16"), py::arg("top_k"), py::arg("top_p"),
        py::arg("top_k_rows") = py::none(), py::arg("top_p_rows") = py::none(),
        py::arg("uniforms") = py::none(), py::arg("seed") = 0, py::arg("offset") = -1,
        py::arg("row_base") = 0, py::arg("temperature") = 1.0);
  m.def("tp_merge", &tp_merge, "vocab-shard exchange over peer memory + merge + sample",
        py::arg("local_cand"), py::arg("bf16"), py::arg("top_k"), py::arg("top_p"), py::arg("recv"),
        py::arg("flags"), py::arg("peer_recv"), py::arg("peer_flags"), py::arg("world"), py::arg("rank"),
        py::arg("epoch"), py::arg("uniforms") = py::none(), py::arg("seed") = 0, py::arg("offset") = -1,
        py::arg("row_base") = 0, py::arg("wait_polls") = 0, py::arg("temperature") = 1.0,
        py::arg("epoch_counter") = py::none());
  m.def("plan", &plan,
        "launch plan (splits, chunks, threads, capacity, maxima/thread, lanes/max, smem, path, workspace)");
  m.attr("NUM_PHASES") = FS_NUM_PHASES;
}
