// g4_noalloc.cu -- attention without any device allocation.
//
// g4_op_attention needs scratch for its per-block softmax partials and takes it from the
// stream-ordered allocator on every call. Some callers cannot allocate at all: a host that has
// already divided device memory between its own pools and forbids any further allocation, a
// process that must never block on or fail in the allocator once it is serving, or an embedding
// (a browser GPU process behind an addon, a plugin inside another runtime) whose allocator belongs
// to someone else. For them this file provides the same operator with its scratch in a
// file-scope device array of fixed size, which the driver places when it loads this library's
// module on a device and which every device that loads the library keeps until the process exits.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/g4.h"
#include "g4_kernels.cuh"

void g4_internal_set_error(const char *msg);

namespace {

// 4 MiB: the per-block partials of g4_op_attention for up to 1,048,576 floats, e.g. one query
// row over 4,096 positions at head_dim 512 (64 blocks x 8 heads x 514 floats = 263,168) or 255
// (row, block) pairs at that head size.
constexpr size_t kScratchFloats = size_t(1) << 20;

static __device__ __align__(256) float g4_attention_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;

// The array's device address per device. Only a successful lookup is kept: a lookup that fails
// (for instance a first call made while the stream is being captured and the module is not yet
// loaded) leaves the slot empty, and the next call tries again.
std::mutex g_scratch_mutex;
float *g_scratch[kMaxDevices] = {};

int set_error(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g4_internal_set_error(buf);
  return code;
}

}  // namespace

// The device address of the scratch array on `device`, looked up with that device current (the
// caller has made it current). Host code must never pass &g4_attention_scratch itself to a
// kernel: on the host that name is only a stand-in, not a device address.
static int scratch_for(int device, float **out) {
  if (device < 0 || device >= kMaxDevices)
    return set_error(G4_ERR_UNSUPPORTED, "device ordinal %d outside the %d supported", device, kMaxDevices);
  std::lock_guard<std::mutex> g(g_scratch_mutex);
  if (!g_scratch[device]) {
    float *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress((void **)&p, g4_attention_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      g4_internal_set_error((std::string("attention scratch set-up failed: ") + cudaGetErrorString(e)).c_str());
      return G4_ERR_CUDA;
    }
    g_scratch[device] = p;
  }
  *out = g_scratch[device];
  return G4_OK;
}

// Device of a device-memory pointer, or -1 when it is not device memory.
static int device_of(const void *p) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return attr.type == cudaMemoryTypeDevice ? attr.device : -1;
}

// Restores the calling thread's current device on every return path.
struct DeviceRestore {
  int dev = -1;
  DeviceRestore() {
    if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  }
  ~DeviceRestore() {
    if (dev >= 0) cudaSetDevice(dev);
  }
};

extern "C" int g4_op_attention_noalloc(const float *q, const float *cache, float *out, int32_t heads,
                                       int32_t head_dim, int32_t q_count, int32_t q_start,
                                       int32_t kv_len, int32_t window, int32_t max_context,
                                       void *stream) {
  if (!q || !cache || !out) return set_error(G4_ERR_INVALID, "g4_op_attention_noalloc: null pointer");
  if (heads != 8) return set_error(G4_ERR_UNSUPPORTED, "the attention kernel is built for 8 query heads, got %d", heads);
  if (head_dim != 256 && head_dim != 512) return set_error(G4_ERR_UNSUPPORTED, "head_dim %d unsupported (256 or 512)", head_dim);
  if (q_count < 1 || q_start < 0 || kv_len < 1 || q_start + q_count > kv_len || kv_len > max_context)
    return set_error(G4_ERR_INVALID, "attention: query rows from %d extend past kv_len %d; store KV before attending", q_start, kv_len);
  const int max_blocks = window > 0 ? (window + 63) / 64 + 1 : (kv_len + 63) / 64;
  const size_t n_o = (size_t)q_count * max_blocks * heads * head_dim;
  const size_t n_ml = (size_t)q_count * max_blocks * heads;
  const size_t need = n_o + 2 * n_ml;
  if (need > kScratchFloats)
    return set_error(G4_ERR_INVALID,
                     "g4_op_attention_noalloc needs %lld floats of scratch; its static array holds %lld "
                     "(use fewer query rows or g4_op_attention)", (long long)need, (long long)kScratchFloats);
  const int dev = device_of(q);
  if (dev < 0) return set_error(G4_ERR_INVALID, "g4_op_attention_noalloc: q is not device memory");
  if (device_of(cache) != dev || device_of(out) != dev)
    return set_error(G4_ERR_INVALID, "g4_op_attention_noalloc: cache and out must be device memory on q's device %d", dev);
  if (stream) {
    int sdev = -1;
    if (cudaStreamGetDevice((cudaStream_t)stream, &sdev) != cudaSuccess || sdev != dev) {
      cudaGetLastError();
      return set_error(G4_ERR_INVALID, "g4_op_attention_noalloc: the stream does not belong to q's device %d", dev);
    }
  }
  DeviceRestore restore;
  if (cudaSetDevice(dev) != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_op_attention_noalloc: cannot make device %d current", dev);
  float *scratch = nullptr;
  int rc = scratch_for(dev, &scratch);
  if (rc) return rc;
  g4::AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.cols = q_count;
  a.heads = heads;
  a.hd = head_dim;
  a.window = window;
  a.max_ctx = max_context;
  a.kv_cap = kv_len;
  a.qr = q;
  a.cache = cache;
  a.seq_stride = 0;
  a.refs.pos_base = q_start;
  a.max_blocks = max_blocks;
  // Every partial a block writes is written before the merge reads it, so nothing needs clearing
  // between calls even though the array keeps the previous call's contents.
  a.part_o = scratch;
  a.part_m = scratch + n_o;
  a.part_l = scratch + n_o + n_ml;
  a.out = out;
  cudaError_t e = g4::launch_attention(a, (cudaStream_t)stream, false);
  if (e != cudaSuccess) {
    g4_internal_set_error((std::string("g4_op_attention_noalloc: ") + cudaGetErrorString(e)).c_str());
    return G4_ERR_CUDA;
  }
  return G4_OK;
}
