// C-ABI plumbing: error reporting, device set-up, memory information, the device error word and
// the host-side integer work of the path (SplitMix64 Rng, synthetic Zipf bytes, Corpus::batch),
// which must be bit-exact with the reference.
#include <cmath>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"

__device__ int g_sj_device_error = 0;

namespace sj {

static thread_local std::string t_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_error = buf;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SJ_OK;
  return fail(SJ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SJ_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int sm_count() {
  static int cached[64];
  static std::once_flag once;
  std::call_once(once, [] {
    for (int& c : cached) c = 0;
  });
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

}  // namespace sj

extern "C" {

int sj_version(void) { return 1; }

const char* sj_last_error(void) { return sj::t_error.c_str(); }

int sj_device_init(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return sj::cuda_check(e, "cudaSetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10)
    return sj::fail(SJ_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device, major,
                    minor);
  sj::sm_count();
  return SJ_OK;
}

int sj_mem_info(size_t* free_bytes, size_t* total_bytes) {
  return sj::cuda_check(cudaMemGetInfo(free_bytes, total_bytes), "cudaMemGetInfo");
}

int sj_device_error(int* code, int clear, void* stream) {
  cudaStream_t s = sj::as_stream(stream);
  int value = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&value, g_sj_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return sj::cuda_check(e, "sj_device_error");
  if (code) *code = value;
  if (clear && value) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_sj_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return sj::cuda_check(e, "sj_device_error clear");
  }
  return SJ_OK;
}

int sj_zero(void* ptr, size_t bytes, void* stream) {
  if (bytes == 0) return SJ_OK;
  if (!ptr) return sj::fail(SJ_ERR_ARGUMENT, "sj_zero: null pointer");
  return sj::zero_async(ptr, bytes, sj::as_stream(stream));
}

// ---------------------------------------------------------------- Rng (crates/sejong-core/src/lib.rs:591-623)
uint64_t sj_rng_next_u64(uint64_t* state) {
  *state += 0x9e3779b97f4a7c15ull;
  uint64_t z = *state;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

static float rng_uniform(uint64_t* state) {
  return static_cast<float>((static_cast<double>(sj_rng_next_u64(state) >> 40) + 0.5) / 16777216.0);
}

uint64_t sj_rng_index(uint64_t* state, uint64_t size) {
  if (size == 0) return 0;
  const uint64_t threshold = (0 - size) % size;
  while (true) {
    const uint64_t x = sj_rng_next_u64(state);
    if (x >= threshold) return x % size;
  }
}

int sj_rng_normal_fill(uint64_t* state, float* out, size_t n, float scale) {
  if (!state || (!out && n)) return sj::fail(SJ_ERR_ARGUMENT, "sj_rng_normal_fill: null pointer");
  const float tau = 6.28318530717958647692f;
  for (size_t i = 0; i < n; ++i) {
    const float a = rng_uniform(state);
    const float b = rng_uniform(state);
    out[i] = std::sqrt(-2.0f * std::log(a)) * std::cos(tau * b) * scale;
  }
  return SJ_OK;
}

int sj_zipf_bytes(uint64_t seed, double s, uint8_t* out, size_t n) {
  if (!out && n) return sj::fail(SJ_ERR_ARGUMENT, "sj_zipf_bytes: null output");
  double cdf[256];
  double total = 0.0;
  for (int k = 0; k < 256; ++k) total += std::pow(static_cast<double>(k + 1), -s);
  double acc = 0.0;
  for (int k = 0; k < 256; ++k) {
    acc += std::pow(static_cast<double>(k + 1), -s) / total;
    cdf[k] = acc;
  }
  uint64_t state = seed;
  for (size_t i = 0; i < n; ++i) {
    const double u = static_cast<double>(rng_uniform(&state));
    int lo = 0, hi = 256;  // first k with cdf[k] >= u
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (cdf[mid] < u)
        lo = mid + 1;
      else
        hi = mid;
    }
    out[i] = static_cast<uint8_t>(lo > 255 ? 255 : lo);
  }
  return SJ_OK;
}

int sj_corpus_batch(const int32_t* tokens, size_t n_tokens, uint64_t* rng_state, int batch, int sequence,
                    int32_t* inputs, int32_t* targets) {
  if (!tokens || !rng_state || !inputs || !targets) return sj::fail(SJ_ERR_ARGUMENT, "sj_corpus_batch: null pointer");
  if (batch <= 0 || sequence <= 0 || n_tokens <= static_cast<size_t>(sequence))
    return sj::fail(SJ_ERR_SHAPE, "corpus is shorter than the training sequence");
  for (int b = 0; b < batch; ++b) {
    const uint64_t start = sj_rng_index(rng_state, n_tokens - static_cast<size_t>(sequence));
    std::memcpy(inputs + static_cast<size_t>(b) * sequence, tokens + start, sizeof(int32_t) * sequence);
    std::memcpy(targets + static_cast<size_t>(b) * sequence, tokens + start + 1, sizeof(int32_t) * sequence);
  }
  return SJ_OK;
}

}  // extern "C"
