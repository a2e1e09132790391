// The C ABI (include/attn_b200.h): argument checks with the reference's error
// conditions, per-device state (SM count, address of the device status word),
// and dispatch to the launchers. No entry point allocates device memory or
// synchronises the host, except attn_device_status which reads the status word.
// The library's own device memory is two module globals, resident on every GPU
// where its kernels are loaded: the status word below and the 32 MiB scratch
// array of attn_paged_decode_noalloc (csrc/decode.cu).
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/attn_b200.h"
#include "common.cuh"
#include "launch.h"

namespace fab {
namespace {

// The status word: one per device that loads the library.
__device__ DeviceStatus g_device_status;

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(ATTN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  DeviceStatus* status = nullptr;
};

std::mutex g_state_mu;
DeviceState g_state[kMaxDevices];

// Per-device set-up on first use; runs with `dev` current.
int device_ctx(cudaStream_t stream, LaunchCtx* ctx) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(ATTN_ERR_CUDA, "device index %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(g_state_mu);
    DeviceState& s = g_state[dev];
    if (!s.ready) {
      int major = 0, minor = 0;
      e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
      if (major != 10 || minor != 0)
        return fail(ATTN_ERR_UNSUPPORTED,
                    "device %d has compute capability %d.%d; this library is built for sm_100a (B200)",
                    dev, major, minor);
      e = cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
      void* addr = nullptr;
      e = cudaGetSymbolAddress(&addr, g_device_status);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status word)");
      s.status = static_cast<DeviceStatus*>(addr);
      s.ready = true;
    }
    ctx->sm_count = s.sm_count;
    ctx->status = s.status;
  }
  ctx->stream = stream;
  ctx->timeout_ns = kDefaultTimeoutNs;
  return ATTN_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_prefill(const char* name, const void* q, const void* k, const void* v, const void* o,
                  int64_t batch, int64_t heads, int64_t seq, int64_t head_dim) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr)
    return fail(ATTN_ERR_INVALID, "%s: null tensor pointer", name);
  if (batch < 0 || heads < 0 || seq < 0)
    return fail(ATTN_ERR_INVALID, "%s: negative size (batch %lld, heads %lld, seq %lld)", name,
                static_cast<long long>(batch), static_cast<long long>(heads),
                static_cast<long long>(seq));
  if (head_dim != 64 && head_dim != 128)
    return fail(ATTN_ERR_UNSUPPORTED, "%s: head_dim must be 64 or 128, got %lld", name,
                static_cast<long long>(head_dim));
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(ATTN_ERR_INVALID, "%s: q, k, v and o must be 16-byte aligned", name);
  if (batch * heads > 0x7fffffffLL || seq > 0x7fffffffLL)
    return fail(ATTN_ERR_UNSUPPORTED, "%s: batch * heads and seq must fit in 31 bits", name);
  return ATTN_OK;
}

}  // namespace
}  // namespace fab

using namespace fab;

extern "C" {

int attn_abi_version(void) { return ATTN_ABI_VERSION; }

const char* attn_last_error(void) { return t_last_error.c_str(); }

int attn_flash_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                   int64_t heads, int64_t seq, int64_t head_dim, int causal, float scale,
                   int64_t block_n, void* stream) {
  int rc = check_prefill("flash_wmma", q, k, v, o, batch, heads, seq, head_dim);
  if (rc != ATTN_OK) return rc;
  if (block_n != 32 && block_n != 64)
    return fail(ATTN_ERR_UNSUPPORTED,
                "flash_wmma: head_dim must be 64 or 128 and block_n 32 or 64 (got block_n %lld)",
                static_cast<long long>(block_n));
  if ((batch * heads) * ((seq + 255) / 256) > 0x7fffffffLL)
    return fail(ATTN_ERR_UNSUPPORTED,
                "flash_wmma: batch * heads * ceil(seq / 256) must fit in 31 bits");
  if (batch * heads == 0 || seq == 0) return ATTN_OK;
  LaunchCtx ctx;
  rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  std::string err;
  cudaError_t e = launch_flash_tc(q, k, v, o, batch * heads, seq, static_cast<int>(head_dim),
                                  causal != 0, scale, ctx, &err);
  if (!err.empty()) return fail(ATTN_ERR_INVALID, "flash_wmma: %s", err.c_str());
  if (e != cudaSuccess) return cuda_fail(e, "flash_wmma launch");
  return ATTN_OK;
}

int attn_flash_simt_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                        int64_t heads, int64_t seq, int64_t head_dim, int causal, float scale,
                        void* stream) {
  int rc = check_prefill("flash_simt", q, k, v, o, batch, heads, seq, head_dim);
  if (rc != ATTN_OK) return rc;
  if (batch * heads > 65535)
    return fail(ATTN_ERR_UNSUPPORTED, "flash_simt: batch * heads must be <= 65535");
  if (batch * heads == 0 || seq == 0) return ATTN_OK;
  LaunchCtx ctx;
  rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = launch_flash_simt(q, k, v, o, batch * heads, seq, static_cast<int>(head_dim),
                                    causal != 0, scale, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "flash_simt launch");
  return ATTN_OK;
}

size_t attn_naive_workspace_bytes(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  return static_cast<size_t>(batch) * heads * seq * seq * sizeof(float);
}

int attn_naive_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                   int64_t heads, int64_t seq, int64_t head_dim, int causal, float scale,
                   void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_prefill("naive_attention", q, k, v, o, batch, heads, seq, head_dim);
  if (rc != ATTN_OK) return rc;
  if (batch * heads > 65535 || seq > 65535 * 8)
    return fail(ATTN_ERR_UNSUPPORTED, "naive_attention: batch * heads <= 65535 and seq <= 524280");
  if (batch * heads == 0 || seq == 0) return ATTN_OK;
  const size_t need = attn_naive_workspace_bytes(batch, heads, seq);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(ATTN_ERR_WORKSPACE, "naive_attention: workspace of %zu bytes (16-byte aligned) needed",
                need);
  LaunchCtx ctx;
  rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = launch_naive(q, k, v, o, static_cast<float*>(workspace), batch * heads, seq,
                               static_cast<int>(head_dim), causal != 0, scale, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "naive_attention launch");
  return ATTN_OK;
}


size_t attn_paged_decode_workspace_bytes(int64_t batch, int64_t num_heads, int64_t head_dim,
                                         int64_t max_context_len, int64_t partition) {
  if (batch <= 0 || num_heads <= 0 || head_dim <= 0 || partition <= 0) return 0;
  return decode_workspace_bytes(batch, num_heads, head_dim, max_context_len, partition);
}

}  // extern "C"

namespace fab {
namespace {

int check_decode(const char* name, const DecodeArgs& a) {
  if (a.q == nullptr || a.k_cache == nullptr || a.v_cache == nullptr ||
      a.block_tables == nullptr || a.context_lens == nullptr)
    return fail(ATTN_ERR_INVALID, "%s: null tensor pointer", name);
  if (a.batch < 0 || a.hq <= 0 || a.hkv <= 0 || a.bs <= 0 || a.num_blocks < 0 ||
      a.max_blocks < 0 || a.max_ctx < 0)
    return fail(ATTN_ERR_INVALID, "%s: negative or zero size", name);
  if (a.hq % a.hkv != 0)
    return fail(ATTN_ERR_INVALID, "num_heads must be a multiple of num_kv_heads");
  if (a.partition <= 0 || a.partition % 256 != 0 || a.partition > 0x40000000LL)
    return fail(ATTN_ERR_INVALID, "partition size must be a positive multiple of 256");
  const int64_t g = a.hq / a.hkv;
  if ((a.d != 64 && a.d != 128) || (g != 1 && g != 2 && g != 4 && g != 8))
    return fail(ATTN_ERR_UNSUPPORTED,
                "paged_decode: head_dim must be 64/128 and num_heads/num_kv_heads in {1,2,4,8}");
  if (a.max_ctx > 0x7fffffffLL || a.max_blocks > 0x7fffffffLL || a.bs > 0x10000 ||
      a.batch * a.hq > 0x7fffffffLL || a.num_blocks > 0x7fffffffLL)
    return fail(ATTN_ERR_UNSUPPORTED, "%s: sizes must fit in 31 bits (block_size <= 65536)", name);
  if (a.max_ctx > a.max_blocks * a.bs)
    return fail(ATTN_ERR_INVALID,
                "%s: max_context_len %lld needs more than max_blocks_per_seq %lld blocks of %lld",
                name, static_cast<long long>(a.max_ctx), static_cast<long long>(a.max_blocks),
                static_cast<long long>(a.bs));
  if (a.max_ctx > 0 && a.num_blocks == 0)
    return fail(ATTN_ERR_INVALID, "%s: empty cache with a non-empty context", name);
  if (!aligned16(a.q) || !aligned16(a.k_cache) || !aligned16(a.v_cache))
    return fail(ATTN_ERR_INVALID, "%s: q and caches must be 16-byte aligned", name);
  const size_t need = decode_workspace_bytes(a.batch, a.hq, a.d, a.max_ctx, a.partition);
  if (a.workspace == nullptr || a.workspace_bytes < need || (reinterpret_cast<uintptr_t>(a.workspace) & 255u))
    return fail(ATTN_ERR_WORKSPACE, "%s: workspace of %zu bytes (256-byte aligned) needed", name, need);
  return ATTN_OK;
}

}  // namespace
}  // namespace fab

extern "C" {

int attn_paged_decode(const void* q, const void* k_cache, const void* v_cache,
                      const int32_t* block_tables, const int32_t* context_lens, void* out,
                      int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                      int64_t block_size, int64_t num_blocks, int64_t max_blocks_per_seq,
                      int64_t max_context_len, float scale, int64_t partition, void* workspace,
                      size_t workspace_bytes, void* stream) {
  DecodeArgs a{q, k_cache, v_cache, block_tables, context_lens, out, nullptr, nullptr, nullptr,
               batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
               max_blocks_per_seq, max_context_len, partition, scale, workspace, workspace_bytes};
  int rc = check_decode("paged_decode", a);
  if (rc != ATTN_OK) return rc;
  if (out == nullptr || !aligned16(out))
    return fail(ATTN_ERR_INVALID, "paged_decode: out must be a 16-byte aligned pointer");
  if (batch == 0) return ATTN_OK;
  LaunchCtx ctx;
  rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = launch_paged_decode(a, false, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
  return ATTN_OK;
}

int attn_paged_decode_partials(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_tables, const int32_t* context_lens,
                               float* o_part, float* m_part, float* l_part, int64_t batch,
                               int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                               int64_t block_size, int64_t num_blocks,
                               int64_t max_blocks_per_seq, int64_t max_context_len, float scale,
                               int64_t partition, void* workspace, size_t workspace_bytes,
                               void* stream) {
  DecodeArgs a{q, k_cache, v_cache, block_tables, context_lens, nullptr, o_part, m_part, l_part,
               batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
               max_blocks_per_seq, max_context_len, partition, scale, workspace, workspace_bytes};
  int rc = check_decode("paged_decode_partials", a);
  if (rc != ATTN_OK) return rc;
  if (o_part == nullptr || m_part == nullptr || l_part == nullptr)
    return fail(ATTN_ERR_INVALID, "paged_decode_partials: null output pointer");
  if (batch == 0) return ATTN_OK;
  LaunchCtx ctx;
  rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = launch_paged_decode(a, true, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode_partials launch");
  return ATTN_OK;
}

int attn_merge_partials(const float* o_parts, const float* m_parts, const float* l_parts,
                        int64_t num_parts, int64_t rows, int64_t head_dim, int64_t o_part_stride,
                        int64_t ml_part_stride, void* out, void* stream) {
  if (o_parts == nullptr || m_parts == nullptr || l_parts == nullptr || out == nullptr)
    return fail(ATTN_ERR_INVALID, "merge_partials: null pointer");
  if (head_dim != 64 && head_dim != 128)
    return fail(ATTN_ERR_UNSUPPORTED, "merge_partials: head_dim must be 64 or 128");
  if (num_parts < 0 || rows < 0 || o_part_stride < 0 || ml_part_stride < 0 ||
      num_parts > 0x7fffffffLL)
    return fail(ATTN_ERR_INVALID, "merge_partials: negative size or stride");
  if (!aligned16(o_parts) || (o_part_stride % 4) != 0 || !aligned16(out))
    return fail(ATTN_ERR_INVALID, "merge_partials: o_parts, its part stride and out must be 16-byte aligned");
  if (rows == 0) return ATTN_OK;
  LaunchCtx ctx;
  int rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = launch_merge(o_parts, m_parts, l_parts, num_parts, rows, head_dim,
                               o_part_stride, ml_part_stride, out, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "merge_partials launch");
  return ATTN_OK;
}

int attn_device_status(uint32_t* code, uint32_t* site) {
  if (code == nullptr || site == nullptr) return fail(ATTN_ERR_INVALID, "device_status: null pointer");
  LaunchCtx ctx;
  int rc = device_ctx(nullptr, &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  DeviceStatus st{0u, 0u};
  e = cudaMemcpy(&st, ctx.status, sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "reading the status word");
  const DeviceStatus zero{0u, 0u};
  e = cudaMemcpy(ctx.status, &zero, sizeof(zero), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the status word");
  *code = st.code;
  *site = st.site;
  return ATTN_OK;
}

int attn_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
  if (timeout_ns == 0 || timeout_ns > 10000000000ull)
    return fail(ATTN_ERR_INVALID, "selftest: timeout must be in (0, 10 s]");
  LaunchCtx ctx;
  int rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = launch_selftest_wait(timeout_ns, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  return ATTN_OK;
}

int attn_exchange_merge_partials(float* const* slots, uint32_t* const* flags, int world, int rank,
                                 uint32_t epoch, int64_t rows, int64_t head_dim,
                                 int64_t slot_stride, void* out, void* stream) {
  if (slots == nullptr || flags == nullptr || out == nullptr)
    return fail(ATTN_ERR_INVALID, "exchange_merge_partials: null pointer");
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return fail(ATTN_ERR_INVALID, "exchange_merge_partials: rank %d of world %d (at most %d)",
                rank, world, kMaxPeers);
  if (head_dim != 64 && head_dim != 128)
    return fail(ATTN_ERR_UNSUPPORTED, "exchange_merge_partials: head_dim must be 64 or 128");
  if (rows < 0 || rows > 0x7fffffffLL || slot_stride < rows * (head_dim + 2) ||
      (slot_stride % 4) != 0)
    return fail(ATTN_ERR_INVALID,
                "exchange_merge_partials: slot_stride must hold rows * (head_dim + 2) floats "
                "and be a multiple of 4");
  for (int q = 0; q < world; ++q)
    if (slots[q] == nullptr || flags[q] == nullptr || !aligned16(slots[q]))
      return fail(ATTN_ERR_INVALID,
                  "exchange_merge_partials: slot %d must be a 16-byte aligned pointer", q);
  if (!aligned16(out))
    return fail(ATTN_ERR_INVALID, "exchange_merge_partials: out must be 16-byte aligned");
  if (rows == 0) return ATTN_OK;
  LaunchCtx ctx;
  int rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = launch_exchange_merge(slots, flags, world, rank, epoch, rows,
                                        static_cast<int>(head_dim), slot_stride, out, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "exchange_merge_partials launch");
  return ATTN_OK;
}

int attn_selftest_exp2(const float* x, float* y_poly, float* y_mufu, float* y_lib, int64_t n,
                       void* stream) {
  if (x == nullptr || y_poly == nullptr || y_mufu == nullptr || y_lib == nullptr)
    return fail(ATTN_ERR_INVALID, "selftest_exp2: null pointer");
  if (n < 0 || n > (int64_t(1) << 31))
    return fail(ATTN_ERR_INVALID, "selftest_exp2: n must be in [0, 2^31]");
  if (n == 0) return ATTN_OK;
  LaunchCtx ctx;
  int rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  cudaError_t e = launch_selftest_exp2(x, y_poly, y_mufu, y_lib, n, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "selftest_exp2 launch");
  return ATTN_OK;
}

int attn_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                              const int32_t* block_tables, const int32_t* context_lens, void* out,
                              int64_t batch, int64_t num_heads, int64_t num_kv_heads,
                              int64_t head_dim, int64_t block_size, int64_t num_blocks,
                              int64_t max_blocks_per_seq, int64_t max_context_len, float scale,
                              int64_t partition, void* stream) {
  // Same argument checks as attn_paged_decode; the workspace fields are a
  // stand-in here and are replaced by the library's fixed scratch array.
  DecodeArgs a{q, k_cache, v_cache, block_tables, context_lens, out, nullptr, nullptr, nullptr,
               batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
               max_blocks_per_seq, max_context_len, partition, scale,
               reinterpret_cast<void*>(static_cast<uintptr_t>(256)), ~static_cast<size_t>(0)};
  int rc = check_decode("paged_decode_noalloc", a);
  if (rc != ATTN_OK) return rc;
  if (out == nullptr || !aligned16(out))
    return fail(ATTN_ERR_INVALID, "paged_decode_noalloc: out must be a 16-byte aligned pointer");
  if (batch == 0) return ATTN_OK;
  LaunchCtx ctx;
  rc = device_ctx(static_cast<cudaStream_t>(stream), &ctx);
  if (rc != ATTN_OK) return rc;
  std::string err;
  cudaError_t e = paged_decode_static_scratch(a, ctx, &err);
  if (!err.empty()) return fail(ATTN_ERR_WORKSPACE, "%s", err.c_str());
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode_noalloc launch");
  return ATTN_OK;
}

}  // extern "C"
