// Context, error reporting and device-memory entry points of libforgecu.so.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>

#include "common.cuh"

namespace fcu {

static thread_local char g_err[1024] = "";
static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char *e = getenv("FORGECU_NO_PDL");
    return !(e && e[0] == '1');
  }();
  return on;
}

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what, const char *file, int line) {
  set_error("CUDA error %d (%s) in %s at %s:%d", (int)e, cudaGetErrorString(e), what, file, line);
  return FCU_ERR_CUDA;
}

int ctx_scratch(fcu_ctx *ctx, size_t bytes, void **out) {
  if (bytes > ctx->scratch_bytes) {
    if (ctx->scratch) {
      // The old buffer may still be read by queued work on this stream.
      FCU_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
      FCU_CHECK_CUDA(cudaFree(ctx->scratch));
      ctx->scratch = nullptr;
      ctx->scratch_bytes = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    FCU_CHECK_CUDA(cudaMalloc(&ctx->scratch, want));
    ctx->scratch_bytes = want;
  }
  *out = ctx->scratch;
  return FCU_OK;
}

}  // namespace fcu

extern "C" {

const char *fcu_last_error(void) { return fcu::g_err; }

const char *fcu_version(void) { return "forgecu 0.1 (sm_100a)"; }

unsigned long long fcu_launch_count(void) { return fcu::g_launches.load(); }

int fcu_ctx_create(int device, fcu_ctx **out) {
  FCU_REQUIRE(out != nullptr, "fcu_ctx_create: null out");
  int n = 0;
  FCU_CHECK_CUDA(cudaGetDeviceCount(&n));
  FCU_REQUIRE(device >= 0 && device < n, "fcu_ctx_create: device %d of %d", device, n);
  FCU_CHECK_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  FCU_CHECK_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) {
    fcu::set_error("fcu_ctx_create: device %d is sm_%d%d; this build targets sm_100a", device,
                   prop.major, prop.minor);
    return FCU_ERR_UNSUPPORTED;
  }
  fcu_ctx *c = new fcu_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  *out = c;
  return FCU_OK;
}

int fcu_ctx_destroy(fcu_ctx *ctx) {
  if (!ctx) return FCU_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  else cudaDeviceSynchronize();
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->rope_tab) cudaFree(ctx->rope_tab);
  delete ctx;
  return FCU_OK;
}

int fcu_ctx_scratch_bytes(const fcu_ctx *ctx, size_t *out) {
  FCU_REQUIRE(ctx && out, "fcu_ctx_scratch_bytes: null argument");
  *out = ctx->scratch_bytes;
  return FCU_OK;
}

int fcu_ctx_set_stream(fcu_ctx *ctx, void *stream) {
  FCU_CTX(ctx);
  ctx->stream = (cudaStream_t)stream;
  return FCU_OK;
}

int fcu_ctx_set_precision(fcu_ctx *ctx, int precision) {
  FCU_CTX(ctx);
  FCU_REQUIRE(precision == FCU_PREC_FP32 || precision == FCU_PREC_FP32_TC || precision == FCU_PREC_BF16,
              "fcu_ctx_set_precision: unknown mode %d", precision);
  ctx->precision = precision;
  return FCU_OK;
}

int fcu_ctx_get_precision(const fcu_ctx *ctx) { return ctx ? ctx->precision : -1; }

int fcu_sync(fcu_ctx *ctx) {
  FCU_CTX(ctx);
  FCU_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  return FCU_OK;
}

int fcu_malloc(fcu_ctx *ctx, size_t bytes, void **out) {
  FCU_CTX(ctx);
  FCU_REQUIRE(out != nullptr, "fcu_malloc: null out");
  FCU_CHECK_CUDA(cudaMalloc(out, bytes ? bytes : 1));
  return FCU_OK;
}

int fcu_free(fcu_ctx *ctx, void *ptr) {
  FCU_CTX(ctx);
  if (ptr) FCU_CHECK_CUDA(cudaFree(ptr));
  return FCU_OK;
}

int fcu_memcpy_h2d(fcu_ctx *ctx, void *dst, const void *src, size_t bytes) {
  FCU_CTX(ctx);
  FCU_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return FCU_OK;
}

int fcu_memcpy_d2h(fcu_ctx *ctx, void *dst, const void *src, size_t bytes) {
  FCU_CTX(ctx);
  FCU_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  FCU_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  return FCU_OK;
}

int fcu_memset_zero(fcu_ctx *ctx, void *dst, size_t bytes) {
  FCU_CTX(ctx);
  FCU_CHECK_CUDA(cudaMemsetAsync(dst, 0, bytes, ctx->stream));
  return FCU_OK;
}

}  // extern "C"
