// asmllm_b200/csrc/capi.cu -- the C ABI of libasmllm.so (declared in include/asmllm.h).
//
// The synchronous entries keep the reference library's names and signatures
// (THRISHAL12345/asmllm build_kernel.py:85-104, src/runtime/threadpool.h:37-102)
// and its calling contract: the caller owns every buffer, y is valid on return
// (src/kernels/arm64/matmul_q4_neon.S returns after its stores).  Pointers may
// be host memory (numpy arrays, as the reference's ctypes callers pass) or
// device memory.  Host buffers are staged through per-device buffers; weights
// registered with asm_weights_register stay resident in HBM.
//
// The reference returns void and has no error channel; here a failure sets a
// per-thread error (asm_get_last_error) and prints one line to stderr.
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/asmllm.h"
#include "decode_persistent.cuh"
#include "matvec.cuh"
#include "tiles.cuh"

using namespace asmllm;

namespace {

// --------------------------------------------------------------------------
// Error channel
// --------------------------------------------------------------------------
thread_local int t_err_code = ASM_OK;
thread_local std::string t_err_msg;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_err_code = code;
  t_err_msg = buf;
  fprintf(stderr, "asmllm: %s\n", buf);
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(ASM_E_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// --------------------------------------------------------------------------
// Pointer classification
//
// Asked of the driver on every call, never cached: an address says nothing
// about the allocation behind it over time.  A pinned buffer can be
// unregistered (cudaHostUnregister / cudaFreeHost) and its address handed out
// again as pageable memory, and a device allocation can be freed and its
// address reused; a cached kind or mapped device address would then send a
// kernel through a dead mapping.  The query costs well under a microsecond
// against the tens of microseconds of a synchronous call.
// --------------------------------------------------------------------------
enum PtrKind { kHostPageable = 0, kHostPinned = 1, kDevice = 2 };

// *mapped: for pinned host memory, its device-visible address (null if not mapped).
PtrKind classify(const void* p, int* device, const void** mapped = nullptr) {
  cudaPointerAttributes a;
  PtrKind k = kHostPageable;
  int dev = -1;
  const void* dptr = nullptr;
  cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();  // unknown pointer: plain host memory
  } else if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
    k = kDevice;
    dev = a.device;
  } else if (a.type == cudaMemoryTypeHost) {
    k = kHostPinned;
    dev = a.device;
    dptr = a.devicePointer;
  }
  if (device) *device = dev;
  if (mapped) *mapped = dptr;
  return k;
}

// --------------------------------------------------------------------------
// Per-device state: a blocking stream (ordered after the legacy default
// stream, which torch uses unless told otherwise) and staging buffers.
// --------------------------------------------------------------------------
struct Buf {
  void* p = nullptr;
  size_t cap = 0;
};

struct DeviceState {
  bool init = false;
  cudaStream_t stream = nullptr;
  Buf dev[5];   // device staging: weights, scales, x, y, Q5_0 high bits
  Buf glue[4];  // device staging of the decode-glue entries' buffers
  Buf host[2];  // pinned host staging: x, y
  Buf image;    // Q8_0 activation image of the synchronous calls
  unsigned* err_word = nullptr;  // mapped pinned word the kernels' error reports also reach
  std::mutex mu;
};

constexpr int kMaxDev = 64;
DeviceState g_state[kMaxDev];
std::mutex g_state_mu;
int g_num_threads = 0;

int get_state(DeviceState** out, int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return set_error(ASM_E_UNSUPPORTED, "device %d out of range", dev);
  DeviceState& st = g_state[dev];
  std::lock_guard<std::mutex> lk(g_state_mu);
  if (!st.init) {
    e = cudaStreamCreateWithFlags(&st.stream, cudaStreamDefault);
    if (e != cudaSuccess) return cuda_error(e, "cudaStreamCreate");
    e = cudaHostAlloc(&st.err_word, sizeof(unsigned), cudaHostAllocMapped);
    if (e != cudaSuccess) return cuda_error(e, "cudaHostAlloc (error word)");
    *st.err_word = 0;
    e = set_device_error_mirror(st.err_word);
    if (e != cudaSuccess) return cuda_error(e, "device error mirror");
    st.init = true;
  }
  *out = &st;
  if (dev_out) *dev_out = dev;
  return ASM_OK;
}

int ensure_dev(Buf& b, size_t bytes) {
  if (b.cap >= bytes) return ASM_OK;
  if (b.p) cudaFree(b.p);
  b.p = nullptr;
  b.cap = 0;
  size_t cap = bytes < 4096 ? 4096 : bytes;
  cudaError_t e = cudaMalloc(&b.p, cap);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc (staging)");
  b.cap = cap;
  return ASM_OK;
}

int ensure_host(Buf& b, size_t bytes) {
  if (b.cap >= bytes) return ASM_OK;
  if (b.p) cudaFreeHost(b.p);
  b.p = nullptr;
  b.cap = 0;
  size_t cap = bytes < 4096 ? 4096 : bytes;
  cudaError_t e = cudaHostAlloc(&b.p, cap, cudaHostAllocDefault);
  if (e != cudaSuccess) return cuda_error(e, "cudaHostAlloc (staging)");
  b.cap = cap;
  return ASM_OK;
}

// --------------------------------------------------------------------------
// Device ranges declared static by the caller (asm_weights_mark_static): the
// kernel that precedes a matvec never writes them, so the matvec may stream
// them before waiting for that kernel (programmatic dependent launch).
// --------------------------------------------------------------------------
std::mutex g_static_mu;
std::map<uintptr_t, uintptr_t> g_static;  // begin -> end

bool is_static(const void* p, size_t bytes) {
  const uintptr_t b = (uintptr_t)p, e = b + bytes;
  std::lock_guard<std::mutex> lk(g_static_mu);
  auto it = g_static.upper_bound(b);
  if (it == g_static.begin()) return false;
  --it;
  return b >= it->first && e <= it->second;
}

// --------------------------------------------------------------------------
// Registered (resident) weights
// --------------------------------------------------------------------------
struct RegEntry {
  const void* host_w = nullptr;
  const float* host_s = nullptr;
  int64_t M = 0, K = 0;
  int fmt = 0;
  int dev = 0;
  void* d_w = nullptr;
  void* d_s = nullptr;
  bool f16 = false;
  bool packed = false;  // d_w holds packed rows (quants then fp16 scales per row); d_s unused
  size_t bytes = 0;
};

std::mutex g_reg_mu;
std::unordered_map<const void*, RegEntry> g_reg;

void free_entry(RegEntry& e) {
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != e.dev) cudaSetDevice(e.dev);
  if (e.d_w) cudaFree(e.d_w);
  if (e.d_s) cudaFree(e.d_s);
  if (cur != e.dev) cudaSetDevice(cur);
  e.d_w = e.d_s = nullptr;
}

size_t weight_bytes(int fmt, int64_t M, int64_t K) {
  return (size_t)M * (size_t)(K / 32) * (fmt == kFmtQ4_0 ? 16u : 32u);
}

int validate(const char* name, const void* w, const void* s, const void* x, const void* y,
             int64_t M, int64_t K) {
  if (M < 0 || K < 0) return set_error(ASM_E_INVALID, "%s: negative size M=%lld K=%lld", name, (long long)M, (long long)K);
  if (K % 32 != 0) return set_error(ASM_E_INVALID, "%s: K=%lld is not a multiple of 32", name, (long long)K);
  if (M > 0x7fffffffLL || K / 32 > 0x7fffffffLL)
    return set_error(ASM_E_UNSUPPORTED, "%s: size too large M=%lld K=%lld", name, (long long)M, (long long)K);
  if (M > 0 && y == nullptr) return set_error(ASM_E_INVALID, "%s: y is NULL", name);
  if (M > 0 && K > 0 && (w == nullptr || s == nullptr || x == nullptr))
    return set_error(ASM_E_INVALID, "%s: NULL input pointer", name);
  return ASM_OK;
}

// The kernels read weights and x with 16-byte vector loads and scales with
// naturally aligned loads; device buffers must be aligned accordingly.
int check_align(const char* name, const void* w, const void* s, size_t s_align, const void* x) {
  if ((uintptr_t)w % 16 != 0)
    return set_error(ASM_E_INVALID, "%s: qweights device pointer is not 16-byte aligned", name);
  if ((uintptr_t)s % s_align != 0)
    return set_error(ASM_E_INVALID, "%s: scales device pointer is not %zu-byte aligned", name, s_align);
  if ((uintptr_t)x % 16 != 0)
    return set_error(ASM_E_INVALID, "%s: x device pointer is not 16-byte aligned", name);
  return ASM_OK;
}

int check_max_k(const char* name, int fmt, bool fp32_act, int64_t K, int dev) {
  const int64_t mk = max_k(fmt, fp32_act, dev);
  if (K > mk)
    return set_error(ASM_E_UNSUPPORTED, "%s: K=%lld exceeds the supported maximum %lld", name,
                     (long long)K, (long long)mk);
  return ASM_OK;
}

// Device view of a caller buffer: the pointer itself when it is device
// memory on `dev`, else a staged copy (host -> device) in `slot`.
int device_in(DeviceState& st, int dev, const void* p, size_t bytes, int slot, const void** out,
              const char* name) {
  int pdev = -1;
  const PtrKind k = classify(p, &pdev);
  if (k == kDevice) {
    if (pdev != dev)
      return set_error(ASM_E_INVALID, "%s: buffer lives on device %d but the current device is %d", name, pdev, dev);
    *out = p;
    return ASM_OK;
  }
  int rc = ensure_dev(st.dev[slot], bytes);
  if (rc) return rc;
  const void* src = p;
  if (k == kHostPageable && slot == 2) {
    // Small activation vectors go through pinned staging (true async DMA).
    rc = ensure_host(st.host[0], bytes);
    if (rc) return rc;
    memcpy(st.host[0].p, p, bytes);
    src = st.host[0].p;
  }
  cudaError_t e = cudaMemcpyAsync(st.dev[slot].p, src, bytes, cudaMemcpyHostToDevice, st.stream);
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyAsync H2D");
  *out = st.dev[slot].p;
  return ASM_OK;
}

// Synchronous Q8_0-activation calls quantize x with a separate pre-pass into a
// per-device image (default) or inside the matvec (option "sync_fused" = 1).
std::atomic<int> g_opt_sync_fused{0};
// Option "sync_map" -- bit 0: pinned host x mapped into the device and read in place by the
// activation pre-pass; bit 1: pinned host y written in place by the matvec.
// A cleared bit stages that buffer with a copy instead.
std::atomic<int> g_opt_sync_map{3};
std::atomic<int> g_opt_xchg_wait_us{0};  // 0 = the default exchange wait limit (about a second)

bool sync_fused() { return g_opt_sync_fused.load() != 0; }

void sync_matvec(const char* name, int fmt, bool fp32_act, const void* w, const float* s,
                 const float* x, float* y, int64_t M, int64_t K) {
  if (validate(name, w, s, x, y, M, K)) return;
  if (M == 0) return;
  DeviceState* stp = nullptr;
  int dev = 0;
  if (get_state(&stp, &dev)) return;
  DeviceState& st = *stp;
  if (check_max_k(name, fmt, fp32_act, K, dev)) return;
  std::lock_guard<std::mutex> lk(st.mu);

  MatvecArgs a;
  a.fmt = fmt;
  a.fp32_act = fp32_act;
  a.M = M;
  a.K = K;

  // Weights: resident copy if registered, else the caller's device buffer or a staged copy.
  bool have_w = false;
  if (K > 0) {
    std::lock_guard<std::mutex> rl(g_reg_mu);
    auto it = g_reg.find(w);
    // A packed registration serves the Q8_0-activation kernels; the fp32-x
    // kernels read two planes, so they stage the host weights instead.
    if (it != g_reg.end() && it->second.host_s == s && it->second.M == M && it->second.K == K &&
        it->second.fmt == fmt && it->second.dev == dev && !(it->second.packed && fp32_act)) {
      a.w = it->second.d_w;
      a.scales = it->second.d_s;
      a.scales_f16 = it->second.f16;
      a.packed = it->second.packed;
      have_w = true;
    }
  }
  if (K > 0 && !have_w) {
    if (device_in(st, dev, w, weight_bytes(fmt, M, K), 0, &a.w, name)) return;
    if (device_in(st, dev, s, (size_t)M * (K / 32) * sizeof(float), 1, &a.scales, name)) return;
  }
  // Library-owned copies (registered or staged) are never written by a kernel;
  // caller device buffers only when declared static.
  a.weights_static = K > 0 && ((a.w != (const void*)w) ||
                               (is_static(w, weight_bytes(fmt, M, K)) &&
                                is_static(s, (size_t)M * (K / 32) * sizeof(float))));
  // Pinned host x and y are used in place (mapped host memory) where only one
  // kernel touches them: the activation pre-pass reads x once, the matvec
  // writes y once -- no staging copies on those calls.
  const bool image_path = !fp32_act && K > 0 && !sync_fused();
  if (K > 0) {
    const void* dx = nullptr;
    const void* xmap = nullptr;
    int xdev = -1;
    if (image_path && (g_opt_sync_map.load() & 1) && classify(x, &xdev, &xmap) == kHostPinned && xdev == dev &&
        xmap && (uintptr_t)xmap % 16 == 0) {
      dx = xmap;
    } else if (device_in(st, dev, x, (size_t)K * sizeof(float), 2, &dx, name)) {
      return;
    }
    a.x = static_cast<const float*>(dx);
    if (check_align(name, a.w, a.scales, a.scales_f16 ? 2 : 4, a.x)) return;
  }

  int ydev = -1;
  const void* ymap = nullptr;
  PtrKind yk = classify(y, &ydev, &ymap);
  const size_t ybytes = (size_t)M * sizeof(float);
  if (yk == kHostPinned && (g_opt_sync_map.load() & 2) && ydev == dev && ymap && (uintptr_t)ymap % 4 == 0) {
    a.y = static_cast<float*>(const_cast<void*>(ymap));
    yk = kDevice;  // written in place: no copy back
  } else if (yk == kDevice) {
    if (ydev != dev) {
      set_error(ASM_E_INVALID, "%s: y lives on device %d but the current device is %d", name, ydev, dev);
      return;
    }
    a.y = y;
  } else {
    if (ensure_dev(st.dev[3], ybytes)) return;
    a.y = static_cast<float*>(st.dev[3].p);
  }

  cudaError_t e = cudaSuccess;
  if (image_path) {
    // Quantize x once into the device's activation image, then the matvec reads it.
    if (ensure_dev(st.image, act_image_bytes(K / 32))) return;
    const size_t sb = (size_t)M * (K / 32) * (a.scales_f16 ? 2 : 4);
    e = launch_act_image(a.x, st.image.p, 1, K, st.stream, a.w, weight_bytes(fmt, M, K) + (a.packed ? sb : 0),
                         a.packed ? nullptr : a.scales, a.packed ? 0 : sb);
    a.image = st.image.p;
  }
  if (e == cudaSuccess) e = launch_matvec(a, st.stream);
  if (e != cudaSuccess) {
    cuda_error(e, name);
    return;
  }
  float* ybounce = nullptr;
  if (yk == kHostPinned) {
    e = cudaMemcpyAsync(y, a.y, ybytes, cudaMemcpyDeviceToHost, st.stream);
  } else if (yk == kHostPageable) {
    if (ensure_host(st.host[1], ybytes)) return;
    ybounce = static_cast<float*>(st.host[1].p);
    e = cudaMemcpyAsync(ybounce, a.y, ybytes, cudaMemcpyDeviceToHost, st.stream);
  }
  if (e != cudaSuccess) {
    cuda_error(e, "cudaMemcpyAsync D2H");
    return;
  }
  e = cudaStreamSynchronize(st.stream);
  if (e != cudaSuccess) {
    cuda_error(e, name);
    return;
  }
  if (*st.err_word) {
    // A kernel reported an error; the device word holds all of its bits
    // (zero if the caller already consumed them with asm_device_error).
    *st.err_word = 0;
    unsigned v = 0;
    e = read_device_error(&v, true);
    if (e != cudaSuccess) {
      cuda_error(e, name);
      return;
    }
    if (v) {
      set_error(ASM_E_CUDA, "%s: a kernel reported device error bits 0x%x (see asm_device_error); y is not valid",
                name, v);
      return;
    }
  }
  if (ybounce) memcpy(y, ybounce, ybytes);
}

// --------------------------------------------------------------------------
// Synchronous decode-glue entries (asm_rmsnorm, asm_rope, asm_softmax,
// asm_attention, asm_silu_hadamard): each buffer is used in place when it is
// device memory of the current device, else staged through a device buffer
// of this device's state -- copied in when the kernel reads it, copied back
// when the kernel writes it -- and the call returns after the copies back.
// --------------------------------------------------------------------------
struct GlueBuf {
  const void* host;
  size_t bytes;
  bool in, out;
  void* dev;
};

template <class Launch>
void glue_call(const char* name, GlueBuf* b, int nb, Launch launch) {
  DeviceState* stp = nullptr;
  int dev = 0;
  if (get_state(&stp, &dev)) return;
  DeviceState& st = *stp;
  std::lock_guard<std::mutex> lk(st.mu);
  bool staged[4] = {};
  for (int i = 0; i < nb; ++i) {
    int pdev = -1;
    if (classify(b[i].host, &pdev) == kDevice) {
      if (pdev != dev) {
        set_error(ASM_E_INVALID, "%s: a buffer lives on device %d but the current device is %d", name, pdev, dev);
        return;
      }
      b[i].dev = const_cast<void*>(b[i].host);
      continue;
    }
    if (ensure_dev(st.glue[i], b[i].bytes)) return;
    b[i].dev = st.glue[i].p;
    staged[i] = true;
    if (b[i].in) {
      const cudaError_t e = cudaMemcpyAsync(b[i].dev, b[i].host, b[i].bytes, cudaMemcpyHostToDevice, st.stream);
      if (e != cudaSuccess) {
        cuda_error(e, name);
        return;
      }
    }
  }
  cudaError_t e = launch(st.stream);
  if (e == cudaErrorInvalidValue || e == cudaErrorNotSupported) {
    set_error(ASM_E_UNSUPPORTED, "%s: size not supported (%s)", name, cudaGetErrorName(e));
    cudaGetLastError();
    return;
  }
  for (int i = 0; i < nb && e == cudaSuccess; ++i)
    if (staged[i] && b[i].out)
      e = cudaMemcpyAsync(const_cast<void*>(b[i].host), b[i].dev, b[i].bytes, cudaMemcpyDeviceToHost, st.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st.stream);
  if (e != cudaSuccess) cuda_error(e, name);
}

// --------------------------------------------------------------------------
// Async entries: device pointers only
// --------------------------------------------------------------------------
int require_device(const char* name, const void* p, const char* what) {
  int pdev = -1;
  if (classify(p, &pdev) != kDevice)
    return set_error(ASM_E_NOT_DEVICE, "%s: %s is not a device pointer", name, what);
  int cur = 0;
  cudaGetDevice(&cur);
  if (pdev != cur)
    return set_error(ASM_E_INVALID, "%s: %s lives on device %d, current device is %d", name, what, pdev, cur);
  return ASM_OK;
}

int async_matvec(const char* name, int fmt, bool fp32_act, bool f16s, const void* w, const void* s,
                 const float* x, float* y, int32_t* isums, int64_t M, int64_t K, void* stream,
                 bool independent = false) {
  int rc = validate(name, w, s, x, y, M, K);
  if (rc) return rc;
  if (M == 0) return ASM_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if ((rc = check_max_k(name, fmt, fp32_act, K, dev))) return rc;
  if ((rc = require_device(name, y, "y"))) return rc;
  if (K > 0) {
    if ((rc = require_device(name, w, "qweights"))) return rc;
    if ((rc = require_device(name, s, "scales"))) return rc;
    if ((rc = require_device(name, x, "x"))) return rc;
  }
  if (isums && (rc = require_device(name, isums, "isums"))) return rc;
  if (K > 0 && (rc = check_align(name, w, s, f16s ? 2 : 4, x))) return rc;
  if (isums && (uintptr_t)isums % 4 != 0) return set_error(ASM_E_INVALID, "%s: isums is not 4-byte aligned", name);
  MatvecArgs a;
  a.fmt = fmt;
  a.fp32_act = fp32_act;
  a.scales_f16 = f16s;
  a.w = w;
  a.scales = s;
  a.x = x;
  a.y = y;
  a.isums = isums;
  a.M = M;
  a.K = K;
  a.weights_static = K > 0 && is_static(w, weight_bytes(fmt, M, K)) &&
                     is_static(s, (size_t)M * (K / 32) * (f16s ? 2 : 4));
  a.act_independent = independent;
  e = launch_matvec(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

// --------------------------------------------------------------------------
// Scratch of the allocation-free entry point (asm_matmul_q4_noalloc_async).
// One activation image of at most kNoAllocMaxK columns: K/32 blocks of 56
// bytes.  Every device that loads this library holds one copy of it until
// the process exits.  In host code `g_noalloc_image` is only a stand-in for
// the symbol: its device address comes from cudaGetSymbolAddress, looked up
// once per device (with that device current) and kept in g_noalloc_addr.
// --------------------------------------------------------------------------
constexpr int64_t kNoAllocMaxK = 32768;
constexpr size_t kNoAllocImageBytes = (size_t)(kNoAllocMaxK / 32) * 56;  // 57344
static __device__ __align__(256) unsigned char g_noalloc_image[kNoAllocImageBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDev];

}  // namespace

// ==========================================================================
// Exported entry points
// ==========================================================================
extern "C" {

ASMLLM_API void asm_matmul_q4(const uint8_t* qweights, const float* scales, const float* x,
                              float* y, int64_t M, int64_t K) {
  sync_matvec("asm_matmul_q4", kFmtQ4_0, false, qweights, scales, x, y, M, K);
}

ASMLLM_API void asm_matmul_q4_avx512(const uint8_t* qweights, const float* scales,
                                     const float* x, float* y, int64_t M, int64_t K) {
  sync_matvec("asm_matmul_q4_avx512", kFmtQ4_0, true, qweights, scales, x, y, M, K);
}

ASMLLM_API void asm_matmul_q4_f32(const uint8_t* qweights, const float* scales, const float* x,
                                  float* y, int64_t M, int64_t K) {
  sync_matvec("asm_matmul_q4_f32", kFmtQ4_0, true, qweights, scales, x, y, M, K);
}

ASMLLM_API void asm_matmul_q8(const int8_t* qweights, const float* scales, const float* x,
                              float* y, int64_t M, int64_t K) {
  sync_matvec("asm_matmul_q8", kFmtQ8_0, true, qweights, scales, x, y, M, K);
}

ASMLLM_API void asm_matmul_q8q8(const int8_t* qweights, const float* scales, const float* x,
                                float* y, int64_t M, int64_t K) {
  sync_matvec("asm_matmul_q8q8", kFmtQ8_0, false, qweights, scales, x, y, M, K);
}

ASMLLM_API void asm_matmul_q4_mt(const uint8_t* qweights, const float* scales, const float* x,
                                 float* y, int64_t M, int64_t K, int num_threads) {
  (void)num_threads;
  sync_matvec("asm_matmul_q4_mt", kFmtQ4_0, false, qweights, scales, x, y, M, K);
}

ASMLLM_API void asm_matmul_q4_avx512_mt(const uint8_t* qweights, const float* scales,
                                        const float* x, float* y, int64_t M, int64_t K,
                                        int num_threads) {
  (void)num_threads;
  sync_matvec("asm_matmul_q4_avx512_mt", kFmtQ4_0, true, qweights, scales, x, y, M, K);
}

ASMLLM_API void asm_matmul_q8_mt(const int8_t* qweights, const float* scales, const float* x,
                                 float* y, int64_t M, int64_t K, int num_threads) {
  (void)num_threads;
  sync_matvec("asm_matmul_q8_mt", kFmtQ8_0, true, qweights, scales, x, y, M, K);
}

// Q5_0 x fp32 (matmul_q5_avx2.asm): host or device pointers, like the other
// synchronous entries (no weight registry for Q5_0: staged per call).
void sync_q5(const char* name, const uint8_t* ql, const uint8_t* qh, const float* s, const float* x, float* y,
             int64_t M, int64_t K) {
  if (validate(name, ql, s, x, y, M, K)) return;
  if (K > 0 && !qh) {
    set_error(ASM_E_INVALID, "%s: null qh", name);
    return;
  }
  if (M == 0) return;
  DeviceState* stp = nullptr;
  int dev = 0;
  if (get_state(&stp, &dev)) return;
  DeviceState& st = *stp;
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (K > 0 && q5_smem_bytes(K) > (size_t)optin) {  // x is staged in shared memory
    set_error(ASM_E_UNSUPPORTED, "%s: K=%lld exceeds the supported maximum %lld", name, (long long)K,
              (long long)(optin / (36 * 4) * 32));
    return;
  }
  std::lock_guard<std::mutex> lk(st.mu);
  const void *dl = nullptr, *dh = nullptr, *ds = nullptr, *dx = nullptr;
  const int64_t nb = K / 32;
  if (K > 0) {
    if (device_in(st, dev, ql, (size_t)M * nb * 16, 0, &dl, name) ||
        device_in(st, dev, s, (size_t)M * nb * sizeof(float), 1, &ds, name) ||
        device_in(st, dev, x, (size_t)K * sizeof(float), 2, &dx, name) ||
        device_in(st, dev, qh, (size_t)M * nb * 4, 4, &dh, name))
      return;
    if ((uintptr_t)dl % 16 || (uintptr_t)dh % 4 || (uintptr_t)ds % 4 || (uintptr_t)dx % 16) {
      set_error(ASM_E_INVALID, "%s: ql/x must be 16-byte, qh/scales 4-byte aligned", name);
      return;
    }
  }
  int ydev = -1;
  const PtrKind yk = classify(y, &ydev);
  const size_t ybytes = (size_t)M * sizeof(float);
  float* dy = nullptr;
  if (yk == kDevice) {
    if (ydev != dev) {
      set_error(ASM_E_INVALID, "%s: y lives on device %d but the current device is %d", name, ydev, dev);
      return;
    }
    dy = y;
  } else {
    if (ensure_dev(st.dev[3], ybytes)) return;
    dy = static_cast<float*>(st.dev[3].p);
  }
  cudaError_t e = launch_q5_matvec(static_cast<const uint8_t*>(dl), static_cast<const uint8_t*>(dh),
                                   static_cast<const float*>(ds), static_cast<const float*>(dx), dy, M, K, st.stream);
  if (e == cudaSuccess && yk != kDevice) e = cudaMemcpyAsync(y, dy, ybytes, cudaMemcpyDeviceToHost, st.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st.stream);
  if (e != cudaSuccess) cuda_error(e, name);
}

ASMLLM_API void asm_matmul_q5(const uint8_t* ql, const uint8_t* qh, const float* scales, const float* x, float* y,
                              int64_t M, int64_t K) {
  sync_q5("asm_matmul_q5", ql, qh, scales, x, y, M, K);
}

ASMLLM_API void asm_matmul_q5_mt(const uint8_t* ql, const uint8_t* qh, const float* scales, const float* x,
                                 float* y, int64_t M, int64_t K, int num_threads) {
  (void)num_threads;
  sync_q5("asm_matmul_q5_mt", ql, qh, scales, x, y, M, K);
}

ASMLLM_API int asm_gemm_image_async(int fmt, const void* qweights, const void* scales_f16, const void* images,
                                    int64_t image_stride, float* y, int64_t M, int64_t N, int64_t K,
                                    void* stream) {
  const char* name = "asm_gemm_image_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0) return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  if (M <= 0 || N <= 0 || K <= 0 || K % 32 || M > INT32_MAX || N > INT32_MAX)
    return set_error(ASM_E_INVALID, "%s: need M, N > 0 and K > 0 a multiple of 32", name);
  if (image_stride < (int64_t)act_image_bytes(K / 32) || image_stride % 16)
    return set_error(ASM_E_INVALID, "%s: image_stride %lld below the image size or not a multiple of 16", name,
                     (long long)image_stride);
  int rc;
  if ((rc = require_device(name, qweights, "qweights")) || (rc = require_device(name, scales_f16, "scales")) ||
      (rc = require_device(name, images, "images")) || (rc = require_device(name, y, "y")))
    return rc;
  if ((uintptr_t)qweights % 16 || (uintptr_t)images % 16 || (uintptr_t)scales_f16 % 2 || (uintptr_t)y % 4)
    return set_error(ASM_E_INVALID, "%s: qweights and images must be 16-byte aligned", name);
  const bool st = is_static(qweights, weight_bytes(fmt, M, K)) && is_static(scales_f16, (size_t)M * (K / 32) * 2);
  const cudaError_t e = launch_q8act_gemm(fmt, qweights, scales_f16, images, (size_t)image_stride, y, M, N, K, st,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_gemm_narrow_async(int fmt, const void* qweights, const void* scales_f16, const void* images,
                                     int64_t image_stride, float* y, int64_t M, int64_t N, int64_t K,
                                     void* stream) {
  const char* name = "asm_gemm_narrow_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0) return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  if (M <= 0 || N <= 0 || K <= 0 || K % 32 || M > INT32_MAX)
    return set_error(ASM_E_INVALID, "%s: need M, N > 0 and K > 0 a multiple of 32", name);
  if (N > kNarrowMaxN)
    return set_error(ASM_E_UNSUPPORTED, "%s: N=%lld tokens (at most %d; use asm_gemm_image_async)", name,
                     (long long)N, kNarrowMaxN);
  if (image_stride < (int64_t)act_image_bytes(K / 32) || image_stride % 16)
    return set_error(ASM_E_INVALID, "%s: image_stride %lld below the image size or not a multiple of 16", name,
                     (long long)image_stride);
  int rc;
  if ((rc = require_device(name, qweights, "qweights")) || (rc = require_device(name, scales_f16, "scales")) ||
      (rc = require_device(name, images, "images")) || (rc = require_device(name, y, "y")))
    return rc;
  if ((uintptr_t)qweights % 16 || (uintptr_t)images % 16 || (uintptr_t)scales_f16 % 2 || (uintptr_t)y % 4)
    return set_error(ASM_E_INVALID, "%s: qweights and images must be 16-byte aligned", name);
  int dev = 0, sms = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if ((size_t)N * ((size_t)(K / 32) * 40 + 127) > (size_t)optin)
    return set_error(ASM_E_UNSUPPORTED, "%s: N=%lld images of K=%lld exceed the shared memory", name, (long long)N,
                     (long long)K);
  const cudaError_t e = launch_gemm_narrow(fmt, qweights, scales_f16, images, (long long)image_stride, y, M, N, K,
                                           sms > 0 ? sms : 1, optin, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int64_t asm_act_tiles_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0 || K % 32 || N > INT32_MAX) return 0;
  return (int64_t)act_tiles_bytes(N, K);
}

ASMLLM_API int asm_act_tiles_from_image_async(const void* images, int64_t image_stride, int64_t N, int64_t K,
                                              void* tiles, void* stream) {
  const char* name = "asm_act_tiles_from_image_async";
  if (N <= 0 || K <= 0 || K % 32 || N > INT32_MAX)
    return set_error(ASM_E_INVALID, "%s: need N > 0 and K > 0 a multiple of 32", name);
  if (image_stride < (int64_t)act_image_bytes(K / 32) || image_stride % 16)
    return set_error(ASM_E_INVALID, "%s: image_stride %lld below the image size or not a multiple of 16", name,
                     (long long)image_stride);
  int rc;
  if ((rc = require_device(name, images, "images")) || (rc = require_device(name, tiles, "tiles"))) return rc;
  if ((uintptr_t)images % 16 || (uintptr_t)tiles % 16)
    return set_error(ASM_E_INVALID, "%s: images and tiles must be 16-byte aligned", name);
  const cudaError_t e =
      launch_act_tiles_from_image(images, (size_t)image_stride, N, K, tiles, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_gemm_tiles_async(int fmt, const void* qweights, const void* scales_f16, const void* tiles,
                                    float* y, int64_t M, int64_t N, int64_t K, void* stream) {
  const char* name = "asm_gemm_tiles_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0) return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  if (M <= 0 || N <= 0 || K <= 0 || K % 32 || M > INT32_MAX || N > INT32_MAX)
    return set_error(ASM_E_INVALID, "%s: need M, N > 0 and K > 0 a multiple of 32", name);
  int rc;
  if ((rc = require_device(name, qweights, "qweights")) || (rc = require_device(name, scales_f16, "scales")) ||
      (rc = require_device(name, tiles, "tiles")) || (rc = require_device(name, y, "y")))
    return rc;
  if ((uintptr_t)qweights % 16 || (uintptr_t)tiles % 16 || (uintptr_t)scales_f16 % 2 || (uintptr_t)y % 4)
    return set_error(ASM_E_INVALID, "%s: qweights and tiles must be 16-byte aligned", name);
  const bool st = is_static(qweights, weight_bytes(fmt, M, K)) && is_static(scales_f16, (size_t)M * (K / 32) * 2);
  const cudaError_t e =
      launch_q8act_gemm_tiles(fmt, qweights, scales_f16, tiles, y, M, N, K, st, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

// ---------------------------------------------------------------------------
// Batched decode glue (batch_decode.cu)
// ---------------------------------------------------------------------------
ASMLLM_API int asm_rows_norm_tiles_async(const asm_rows_t* d, void* stream) {
  const char* name = "asm_rows_norm_tiles_async";
  if (!d) return set_error(ASM_E_INVALID, "%s: null descriptor", name);
  if (d->rows <= 0 || d->dim <= 0 || d->dim % 32)
    return set_error(ASM_E_INVALID, "%s: need rows > 0 and dim a positive multiple of 32", name);
  if ((size_t)d->dim * sizeof(float) > 200 * 1024) return set_error(ASM_E_UNSUPPORTED, "%s: dim too large", name);
  int rc;
  if ((rc = require_device(name, d->x, "x")) || (rc = require_device(name, d->tiles, "tiles"))) return rc;
  if (d->delta && (rc = require_device(name, d->delta, "delta"))) return rc;
  if (d->norm_w && (rc = require_device(name, d->norm_w, "norm_w"))) return rc;
  if (d->embed) {
    if ((rc = require_device(name, d->embed, "embed")) || (rc = require_device(name, d->tokens, "tokens")) ||
        (rc = require_device(name, d->pos, "pos")))
      return rc;
    if (d->max_tokens <= 0 || d->vocab <= 0)
      return set_error(ASM_E_INVALID, "%s: embed needs max_tokens and vocab", name);
  }
  if ((uintptr_t)d->x % 16 || (uintptr_t)d->tiles % 16 || (uintptr_t)d->delta % 16 || (uintptr_t)d->norm_w % 16 ||
      (uintptr_t)d->embed % 16)
    return set_error(ASM_E_INVALID, "%s: misaligned buffer", name);
  RowsArgs a;
  a.rows = d->rows;
  a.dim = d->dim;
  a.x = d->x;
  a.delta = d->delta;
  a.embed = d->embed;
  a.tokens = d->tokens;
  a.pos = d->pos;
  a.max_tokens = d->max_tokens;
  a.vocab = d->vocab;
  a.norm_w = d->norm_w;
  a.eps = d->eps;
  a.tiles = d->tiles;
  a.np = act_tiles_tokens(d->rows);
  const cudaError_t e = launch_rows_norm_tiles(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_rows_swiglu_tiles_async(const float* gu, int32_t rows, int32_t ffn, void* tiles, void* stream) {
  const char* name = "asm_rows_swiglu_tiles_async";
  if (rows <= 0 || ffn <= 0 || ffn % 32) return set_error(ASM_E_INVALID, "%s: need ffn a positive multiple of 32", name);
  if ((size_t)ffn * sizeof(float) > 200 * 1024) return set_error(ASM_E_UNSUPPORTED, "%s: ffn too large", name);
  int rc;
  if ((rc = require_device(name, gu, "gu")) || (rc = require_device(name, tiles, "tiles"))) return rc;
  if ((uintptr_t)gu % 16 || (uintptr_t)tiles % 16) return set_error(ASM_E_INVALID, "%s: misaligned buffer", name);
  const cudaError_t e = launch_rows_swiglu_tiles(gu, rows, ffn, tiles, act_tiles_tokens(rows),
                                                 static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_attention_batch_async(const float* qkv, int64_t qkv_stride, void* k_cache, void* v_cache,
                                         int64_t cache_stride, const float* rope_cs, const int32_t* pos, void* tiles,
                                         int32_t rows, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                         int32_t ctx, float sqrt_head_dim, void* stream) {
  const char* name = "asm_attention_batch_async";
  if (head_dim != 128) return set_error(ASM_E_UNSUPPORTED, "%s: head_dim %d (only 128)", name, head_dim);
  if (rows <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || ctx <= 0)
    return set_error(ASM_E_INVALID, "%s: need rows > 0, n_heads a multiple of n_kv_heads and ctx > 0", name);
  if (qkv_stride < (int64_t)(n_heads + 2 * n_kv_heads) * head_dim || qkv_stride % 4 ||
      cache_stride < (int64_t)ctx * n_kv_heads * head_dim || cache_stride % 8)
    return set_error(ASM_E_INVALID, "%s: qkv_stride or cache_stride too small or misaligned", name);
  int rc;
  if ((rc = require_device(name, qkv, "qkv")) || (rc = require_device(name, k_cache, "k_cache")) ||
      (rc = require_device(name, v_cache, "v_cache")) || (rc = require_device(name, rope_cs, "rope_cs")) ||
      (rc = require_device(name, pos, "pos")) || (rc = require_device(name, tiles, "tiles")))
    return rc;
  if ((uintptr_t)qkv % 16 || (uintptr_t)k_cache % 16 || (uintptr_t)v_cache % 16 || (uintptr_t)rope_cs % 8 ||
      (uintptr_t)tiles % 16)
    return set_error(ASM_E_INVALID, "%s: misaligned buffer", name);
  const cudaError_t e = launch_attention_batch(qkv, (size_t)qkv_stride, k_cache, v_cache, (size_t)cache_stride,
                                               rope_cs, pos, tiles, act_tiles_tokens(rows), rows, n_heads, n_kv_heads,
                                               head_dim, ctx, sqrt_head_dim, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported) return set_error(ASM_E_UNSUPPORTED, "%s: ctx %d too long for shared memory", name, ctx);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_rows_argmax_async(const float* logits, int32_t rows, int32_t n, int64_t stride, int32_t offset,
                                     int64_t* keys, void* stream) {
  const char* name = "asm_rows_argmax_async";
  if (rows <= 0 || n <= 0 || stride < n || offset < 0)
    return set_error(ASM_E_INVALID, "%s: need rows, n > 0, stride >= n, offset >= 0", name);
  int rc;
  if ((rc = require_device(name, logits, "logits")) || (rc = require_device(name, keys, "keys"))) return rc;
  const cudaError_t e = launch_rows_argmax(logits, rows, n, (size_t)stride, offset, reinterpret_cast<long long*>(keys),
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_rows_advance_async(const int64_t* keys, int32_t rows, int32_t* tokens, int32_t max_tokens,
                                      int32_t* pos, int32_t n_prompt, void* stream) {
  const char* name = "asm_rows_advance_async";
  if (rows <= 0 || max_tokens <= 0) return set_error(ASM_E_INVALID, "%s: need rows, max_tokens > 0", name);
  int rc;
  if ((rc = require_device(name, keys, "keys")) || (rc = require_device(name, tokens, "tokens")) ||
      (rc = require_device(name, pos, "pos")))
    return rc;
  const cudaError_t e = launch_rows_advance(reinterpret_cast<const long long*>(keys), rows, tokens, max_tokens, pos,
                                            n_prompt, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_matmul_q5_async(const uint8_t* ql, const uint8_t* qh, const float* scales, const float* x,
                                   float* y, int64_t M, int64_t K, void* stream) {
  const char* name = "asm_matmul_q5_async";
  int rc = validate(name, ql, scales, x, y, M, K);
  if (rc) return rc;
  if (M == 0) return ASM_OK;
  if ((rc = require_device(name, y, "y"))) return rc;
  if (K > 0) {
    if ((rc = require_device(name, ql, "ql")) || (rc = require_device(name, qh, "qh")) ||
        (rc = require_device(name, scales, "scales")) || (rc = require_device(name, x, "x")))
      return rc;
    if ((uintptr_t)ql % 16 || (uintptr_t)qh % 4 || (uintptr_t)scales % 4 || (uintptr_t)x % 16)
      return set_error(ASM_E_INVALID, "%s: ql/x must be 16-byte, qh/scales 4-byte aligned", name);
  }
  const cudaError_t e = launch_q5_matvec(ql, qh, scales, x, y, M, K, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue) return set_error(ASM_E_UNSUPPORTED, "%s: K=%lld too large", name, (long long)K);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API void asm_threadpool_dispatch_q5(const uint8_t* ql, const uint8_t* qh, const float* scales,
                                           const float* x, float* y, int64_t M, int64_t K) {
  sync_q5("asm_threadpool_dispatch_q5", ql, qh, scales, x, y, M, K);
}

ASMLLM_API void asm_rmsnorm(const float* x, const float* weight, float* y, int64_t dim, float eps) {
  const char* name = "asm_rmsnorm";
  if (dim <= 0 || dim > glue_max_len()) {
    set_error(dim < 0 ? ASM_E_INVALID : ASM_E_UNSUPPORTED, "%s: dim=%lld out of range (1..%lld)", name,
              (long long)dim, (long long)glue_max_len());
    return;
  }
  if (!x || !weight || !y) {
    set_error(ASM_E_INVALID, "%s: NULL pointer", name);
    return;
  }
  const size_t nb = (size_t)dim * 4;
  GlueBuf b[3] = {{x, nb, true, false, nullptr}, {weight, nb, true, false, nullptr}, {y, nb, false, true, nullptr}};
  glue_call(name, b, 3, [&](cudaStream_t s) {
    return launch_rmsnorm(static_cast<const float*>(b[0].dev), static_cast<const float*>(b[1].dev),
                          static_cast<float*>(b[2].dev), dim, eps, s);
  });
}

ASMLLM_API void asm_rope(float* q, float* k, int64_t head_dim, int64_t pos, float theta) {
  const char* name = "asm_rope";
  if (head_dim <= 0 || head_dim % 2 || head_dim > glue_max_len() || pos < 0) {
    set_error(ASM_E_INVALID, "%s: head_dim=%lld must be positive and even, pos=%lld non-negative", name,
              (long long)head_dim, (long long)pos);
    return;
  }
  if (!q || !k) {
    set_error(ASM_E_INVALID, "%s: NULL pointer", name);
    return;
  }
  const size_t nb = (size_t)head_dim * 4;
  GlueBuf b[2] = {{q, nb, true, true, nullptr}, {k, nb, true, true, nullptr}};
  glue_call(name, b, 2, [&](cudaStream_t s) {
    return launch_rope(static_cast<float*>(b[0].dev), static_cast<float*>(b[1].dev), head_dim, pos, theta, s);
  });
}

ASMLLM_API void asm_softmax(const float* x, float* y, int64_t n) {
  const char* name = "asm_softmax";
  if (n <= 0 || n > glue_max_len()) {
    set_error(n < 0 ? ASM_E_INVALID : ASM_E_UNSUPPORTED, "%s: n=%lld out of range (1..%lld)", name, (long long)n,
              (long long)glue_max_len());
    return;
  }
  if (!x || !y) {
    set_error(ASM_E_INVALID, "%s: NULL pointer", name);
    return;
  }
  const size_t nb = (size_t)n * 4;
  GlueBuf b[2] = {{x, nb, true, false, nullptr}, {y, nb, false, true, nullptr}};
  glue_call(name, b, 2, [&](cudaStream_t s) {
    return launch_softmax(static_cast<const float*>(b[0].dev), static_cast<float*>(b[1].dev), n, s);
  });
}

ASMLLM_API void asm_attention(const float* q, const float* k, const float* v, float* y, int64_t seq_len,
                              int64_t head_dim, float scale) {
  const char* name = "asm_attention";
  if (seq_len <= 0 || head_dim <= 0 || seq_len > glue_max_len() || head_dim > glue_max_len()) {
    set_error(ASM_E_INVALID, "%s: seq_len=%lld and head_dim=%lld must be positive", name, (long long)seq_len,
              (long long)head_dim);
    return;
  }
  if (!q || !k || !v || !y) {
    set_error(ASM_E_INVALID, "%s: NULL pointer", name);
    return;
  }
  const size_t nb = (size_t)seq_len * (size_t)head_dim * 4;
  GlueBuf b[4] = {{q, nb, true, false, nullptr}, {k, nb, true, false, nullptr}, {v, nb, true, false, nullptr},
                  {y, nb, false, true, nullptr}};
  glue_call(name, b, 4, [&](cudaStream_t s) {
    return launch_attention(static_cast<const float*>(b[0].dev), static_cast<const float*>(b[1].dev),
                            static_cast<const float*>(b[2].dev), static_cast<float*>(b[3].dev), seq_len, head_dim,
                            scale, s);
  });
}

ASMLLM_API void asm_silu_hadamard(float* gate, const float* up, int64_t n) {
  const char* name = "asm_silu_hadamard";
  if (n < 0) {
    set_error(ASM_E_INVALID, "%s: n=%lld is negative", name, (long long)n);
    return;
  }
  if (n == 0) return;
  if (!gate || !up) {
    set_error(ASM_E_INVALID, "%s: NULL pointer", name);
    return;
  }
  const size_t nb = (size_t)n * 4;
  GlueBuf b[2] = {{gate, nb, true, true, nullptr}, {up, nb, true, false, nullptr}};
  glue_call(name, b, 2, [&](cudaStream_t s) {
    return launch_silu_hadamard(static_cast<float*>(b[0].dev), static_cast<const float*>(b[1].dev), n, s);
  });
}

ASMLLM_API void asm_threadpool_dispatch_q8(const int8_t* qweights, const float* scales,
                                           const float* x, float* y, int64_t M, int64_t K) {
  sync_matvec("asm_threadpool_dispatch_q8", kFmtQ8_0, true, qweights, scales, x, y, M, K);
}

ASMLLM_API void asm_threadpool_init(int num_threads) {
  g_num_threads = num_threads;
  DeviceState* st = nullptr;
  get_state(&st, nullptr);
}

ASMLLM_API void asm_threadpool_shutdown(void) {
  {
    std::lock_guard<std::mutex> rl(g_reg_mu);
    for (auto& kv : g_reg) free_entry(kv.second);
    g_reg.clear();
  }
  int cur = 0;
  cudaGetDevice(&cur);
  for (int d = 0; d < kMaxDev; ++d) {
    DeviceState& st = g_state[d];
    std::lock_guard<std::mutex> lk(st.mu);
    if (!st.init) continue;
    cudaSetDevice(d);
    cudaStreamSynchronize(st.stream);
    for (auto& b : st.dev) {
      if (b.p) cudaFree(b.p);
      b = Buf();
    }
    for (auto& b : st.host) {
      if (b.p) cudaFreeHost(b.p);
      b = Buf();
    }
    if (st.image.p) cudaFree(st.image.p);
    st.image = Buf();
    for (auto& b : st.glue) {
      if (b.p) cudaFree(b.p);
      b = Buf();
    }
    cudaStreamDestroy(st.stream);
    st.stream = nullptr;
    set_device_error_mirror(nullptr);
    if (st.err_word) cudaFreeHost(st.err_word);
    st.err_word = nullptr;
    st.init = false;
  }
  scratch_trim();
  cudaSetDevice(cur);
  g_num_threads = 0;
}

ASMLLM_API int asm_threadpool_get_num_threads(void) { return g_num_threads; }

ASMLLM_API int asm_pointer_kind(const void* p, int* device) {
  int dev = -1;
  const PtrKind k = classify(p, &dev);
  if (device) *device = dev;
  return (int)k;
}

ASMLLM_API void asm_quantize_q8_0(const float* x, int8_t* xq, float* xd, int64_t K) {
  const char* name = "asm_quantize_q8_0";
  if (K < 0 || K % 32 != 0) {
    set_error(ASM_E_INVALID, "%s: K=%lld must be a non-negative multiple of 32", name, (long long)K);
    return;
  }
  if (K == 0) return;
  if (!x || !xq || !xd) {
    set_error(ASM_E_INVALID, "%s: NULL pointer", name);
    return;
  }
  DeviceState* stp = nullptr;
  int dev = 0;
  if (get_state(&stp, &dev)) return;
  DeviceState& st = *stp;
  std::lock_guard<std::mutex> lk(st.mu);
  const int64_t nb = K / 32;
  const void* dx = nullptr;
  if (device_in(st, dev, x, (size_t)K * 4, 2, &dx, name)) return;
  int qdev = -1, ddev = -1;
  const PtrKind qk = classify(xq, &qdev), dk = classify(xd, &ddev);
  int8_t* dq = xq;
  float* dd = xd;
  // Outputs that are host memory are produced in the weight staging slots.
  if (qk != kDevice) {
    if (ensure_dev(st.dev[0], (size_t)K)) return;
    dq = static_cast<int8_t*>(st.dev[0].p);
  }
  if (dk != kDevice) {
    if (ensure_dev(st.dev[1], (size_t)nb * 4)) return;
    dd = static_cast<float*>(st.dev[1].p);
  }
  cudaError_t e = launch_quantize(static_cast<const float*>(dx), dq, dd, nb, st.stream);
  if (e != cudaSuccess) {
    cuda_error(e, name);
    return;
  }
  if (qk != kDevice) e = cudaMemcpyAsync(xq, dq, (size_t)K, cudaMemcpyDeviceToHost, st.stream);
  if (e == cudaSuccess && dk != kDevice)
    e = cudaMemcpyAsync(xd, dd, (size_t)nb * 4, cudaMemcpyDeviceToHost, st.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st.stream);
  if (e != cudaSuccess) cuda_error(e, name);
}

ASMLLM_API int asm_weights_register(const void* qweights, const float* scales, int64_t M,
                                    int64_t K, int fmt) {
  const char* name = "asm_weights_register";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0)
    return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 (Q4_0) or 8 (Q8_0)", name, fmt);
  if (M <= 0 || K <= 0) return set_error(ASM_E_INVALID, "%s: M and K must be positive", name);
  int rc = validate(name, qweights, scales, scales, scales, M, K);
  if (rc) return rc;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (classify(qweights, nullptr) == kDevice || classify(scales, nullptr) == kDevice)
    return set_error(ASM_E_INVALID, "%s: expects host buffers (device buffers are already resident)", name);
  asm_weights_unregister(qweights);

  const size_t wb = weight_bytes(fmt, M, K);
  const size_t n = (size_t)M * (size_t)(K / 32);
  // fp16 scales when every scale survives the round trip exactly.
  bool f16 = true;
  std::vector<__half> hs(n);
  for (size_t i = 0; i < n; ++i) {
    hs[i] = __float2half_rn(scales[i]);
    const float back = __half2float(hs[i]);
    if (!(back == scales[i]) && !(back != back && scales[i] != scales[i])) {
      f16 = false;
      break;
    }
  }
  RegEntry r;
  r.host_w = qweights;
  r.host_s = scales;
  r.M = M;
  r.K = K;
  r.fmt = fmt;
  r.dev = dev;
  r.f16 = f16;
  const size_t sb = n * (f16 ? 2 : 4);
  // fp16 scales and K/32 a multiple of 8: one packed plane (each row's quants,
  // then its scales), streamed one copy per stage.
  const int64_t nb = K / 32;
  r.packed = f16 && nb % 8 == 0;
  if (r.packed) {
    const size_t qrow = (size_t)nb * (fmt == kFmtQ4_0 ? 16 : 32), srow = (size_t)nb * 2;
    std::vector<unsigned char> rows((size_t)M * (qrow + srow));
    for (int64_t i = 0; i < M; ++i) {
      memcpy(rows.data() + (size_t)i * (qrow + srow), static_cast<const unsigned char*>(qweights) + (size_t)i * qrow,
             qrow);
      memcpy(rows.data() + (size_t)i * (qrow + srow) + qrow, hs.data() + (size_t)i * nb, srow);
    }
    if ((e = cudaMalloc(&r.d_w, rows.size())) != cudaSuccess) return cuda_error(e, "cudaMalloc (weights)");
    e = cudaMemcpy(r.d_w, rows.data(), rows.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      free_entry(r);
      return cuda_error(e, "cudaMemcpy (register)");
    }
    r.bytes = rows.size();
    std::lock_guard<std::mutex> rl(g_reg_mu);
    g_reg[qweights] = r;
    return ASM_OK;
  }
  if ((e = cudaMalloc(&r.d_w, wb)) != cudaSuccess) return cuda_error(e, "cudaMalloc (weights)");
  if ((e = cudaMalloc(&r.d_s, sb)) != cudaSuccess) {
    cudaFree(r.d_w);
    return cuda_error(e, "cudaMalloc (scales)");
  }
  e = cudaMemcpy(r.d_w, qweights, wb, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(r.d_s, f16 ? (const void*)hs.data() : (const void*)scales, sb, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    free_entry(r);
    return cuda_error(e, "cudaMemcpy (register)");
  }
  r.bytes = wb + sb;
  std::lock_guard<std::mutex> rl(g_reg_mu);
  g_reg[qweights] = r;
  return ASM_OK;
}

ASMLLM_API int asm_weights_unregister(const void* qweights) {
  std::lock_guard<std::mutex> rl(g_reg_mu);
  auto it = g_reg.find(qweights);
  if (it == g_reg.end()) return ASM_OK;
  // Calls on the library streams that may still read the copy finish first.
  for (int d = 0; d < kMaxDev; ++d)
    if (g_state[d].init) cudaStreamSynchronize(g_state[d].stream);
  free_entry(it->second);
  g_reg.erase(it);
  return ASM_OK;
}

ASMLLM_API int64_t asm_weights_resident_bytes(int* count) {
  std::lock_guard<std::mutex> rl(g_reg_mu);
  int64_t total = 0;
  for (auto& kv : g_reg) total += (int64_t)kv.second.bytes;
  if (count) *count = (int)g_reg.size();
  return total;
}

ASMLLM_API int asm_get_last_error(char* buf, size_t n) {
  const int code = t_err_code;
  if (buf && n) {
    const size_t len = t_err_msg.size() < n - 1 ? t_err_msg.size() : n - 1;
    memcpy(buf, t_err_msg.data(), len);
    buf[len] = '\0';
  }
  t_err_code = ASM_OK;
  t_err_msg.clear();
  return code;
}

ASMLLM_API int asm_matmul_q4_async(const uint8_t* qweights, const float* scales, const float* x,
                                   float* y, int64_t M, int64_t K, void* stream) {
  return async_matvec("asm_matmul_q4_async", kFmtQ4_0, false, false, qweights, scales, x, y,
                      nullptr, M, K, stream);
}

ASMLLM_API int asm_matmul_q4_f16s_async(const uint8_t* qweights, const uint16_t* scales_f16,
                                        const float* x, float* y, int64_t M, int64_t K,
                                        void* stream) {
  return async_matvec("asm_matmul_q4_f16s_async", kFmtQ4_0, false, true, qweights, scales_f16, x,
                      y, nullptr, M, K, stream);
}

ASMLLM_API int asm_matvec_ex_async(int fmt, const void* qweights, const void* scales, int scales_are_f16,
                                   const float* x, float* y, int64_t M, int64_t K, unsigned flags, void* stream) {
  const char* name = "asm_matvec_ex_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0) return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  if (flags & ~(unsigned)ASM_MV_INDEPENDENT) return set_error(ASM_E_INVALID, "%s: unknown flags 0x%x", name, flags);
  return async_matvec(name, fmt, false, scales_are_f16 != 0, qweights, scales, x, y, nullptr, M, K, stream,
                      (flags & ASM_MV_INDEPENDENT) != 0);
}

ASMLLM_API int asm_launch_floor_async(int32_t n, int32_t pdl, int32_t wait, void* stream) {
  if (n < 0) return set_error(ASM_E_INVALID, "asm_launch_floor_async: n=%d is negative", n);
  const cudaError_t e = launch_floor_chain(n, pdl != 0, wait != 0, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, "asm_launch_floor_async");
  return ASM_OK;
}

ASMLLM_API int64_t asm_packed_row_bytes(int fmt, int64_t K) {
  if ((fmt != kFmtQ4_0 && fmt != kFmtQ8_0) || K <= 0 || K % 256 != 0) return -1;
  return (K / 32) * ((fmt == kFmtQ4_0 ? 16 : 32) + 2);
}

ASMLLM_API int asm_pack_rows_async(int fmt, const void* qweights, const uint16_t* scales_f16, void* packed, int64_t M,
                                   int64_t K, void* stream) {
  const char* name = "asm_pack_rows_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0) return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  if (M <= 0 || K <= 0 || K % 256 != 0 || M > INT32_MAX)
    return set_error(ASM_E_INVALID, "%s: need M > 0 and K > 0 a multiple of 256", name);
  int rc;
  if ((rc = require_device(name, qweights, "qweights")) || (rc = require_device(name, scales_f16, "scales")) ||
      (rc = require_device(name, packed, "packed")))
    return rc;
  if ((uintptr_t)qweights % 16 || (uintptr_t)scales_f16 % 16 || (uintptr_t)packed % 16)
    return set_error(ASM_E_INVALID, "%s: buffers must be 16-byte aligned", name);
  const cudaError_t e = launch_pack_rows(fmt, qweights, scales_f16, packed, M, K, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_matvec_packed_async(int fmt, const void* packed, const float* x, float* y, int64_t M, int64_t K,
                                       unsigned flags, void* stream) {
  const char* name = "asm_matvec_packed_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0) return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  if (flags & ~(unsigned)ASM_MV_INDEPENDENT) return set_error(ASM_E_INVALID, "%s: unknown flags 0x%x", name, flags);
  int rc = validate(name, packed, packed, x, y, M, K);
  if (rc) return rc;
  if (M == 0) return ASM_OK;
  if (K % 256 != 0) return set_error(ASM_E_INVALID, "%s: K=%lld is not a multiple of 256", name, (long long)K);
  if ((rc = require_device(name, packed, "packed")) || (rc = require_device(name, x, "x")) ||
      (rc = require_device(name, y, "y")))
    return rc;
  if ((uintptr_t)packed % 16 || (uintptr_t)x % 16)
    return set_error(ASM_E_INVALID, "%s: packed and x must be 16-byte aligned", name);
  MatvecArgs a;
  a.fmt = fmt;
  a.packed = true;
  a.scales_f16 = true;
  a.w = packed;
  a.x = x;
  a.y = y;
  a.M = M;
  a.K = K;
  a.weights_static = K > 0 && is_static(packed, (size_t)M * (size_t)asm_packed_row_bytes(fmt, K));
  a.act_independent = (flags & ASM_MV_INDEPENDENT) != 0;
  const cudaError_t e = launch_matvec(a, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)
    return set_error(ASM_E_UNSUPPORTED, "%s: no bulk-copy plan for K=%lld (or the tma option is off)", name,
                     (long long)K);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_matvec_rowsplit_async(int fmt, const void* qweights, const uint16_t* scales_f16, const float* x,
                                         float* y_full, int64_t M, int64_t K, int32_t tp, int32_t rank,
                                         void* const* xchg, uint32_t* seq, unsigned flags, void* stream) {
  const char* name = "asm_matvec_rowsplit_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0) return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  if (flags & ~(unsigned)(ASM_MV_INDEPENDENT | ASM_MV_PACKED))
    return set_error(ASM_E_INVALID, "%s: unknown flags 0x%x", name, flags);
  if (tp < 1 || tp > kMaxTp || rank < 0 || rank >= tp)
    return set_error(ASM_E_INVALID, "%s: tp=%d rank=%d (need 1 <= tp <= %d, 0 <= rank < tp)", name, tp, rank, kMaxTp);
  const bool packed = (flags & ASM_MV_PACKED) != 0;
  int rc = validate(name, qweights, packed ? qweights : (const void*)scales_f16, x, y_full, M, K);
  if (rc) return rc;
  if (M == 0) return ASM_OK;
  if (packed && K % 256 != 0) return set_error(ASM_E_INVALID, "%s: K=%lld is not a multiple of 256", name, (long long)K);
  if ((rc = require_device(name, qweights, "qweights")) || (!packed && (rc = require_device(name, scales_f16, "scales"))) ||
      (rc = require_device(name, x, "x")) || (rc = require_device(name, y_full, "y_full")))
    return rc;
  if (!seq) return set_error(ASM_E_INVALID, "%s: seq is null", name);
  if ((rc = require_device(name, seq, "seq"))) return rc;
  MvFuse fz;
  fz.tp = tp;
  fz.tp_rank = rank;
  fz.xchg_rows = (int)M;
  fz.ar_seq = seq;
  for (int r = 0; r < tp; ++r) {
    if (r == rank) continue;
    if (!xchg || !xchg[r]) return set_error(ASM_E_INVALID, "%s: gather buffer of rank %d is null", name, r);
    fz.xchg[r] = static_cast<unsigned long long*>(xchg[r]);
  }
  if (M > INT32_MAX / kMaxTp) return set_error(ASM_E_INVALID, "%s: M=%lld too large", name, (long long)M);
  MatvecArgs a;
  a.fmt = fmt;
  a.packed = packed;
  a.scales_f16 = true;
  a.w = qweights;
  a.scales = packed ? nullptr : scales_f16;
  a.x = x;
  a.y = y_full;
  a.M = M;
  a.K = K;
  a.epi = kEpiGather;
  a.fuse = &fz;
  const size_t wbytes = packed ? (size_t)M * (size_t)asm_packed_row_bytes(fmt, K)
                               : (size_t)M * (size_t)(K / 32) * (fmt == kFmtQ4_0 ? 16 : 32);
  a.weights_static = is_static(qweights, wbytes);
  a.act_independent = (flags & ASM_MV_INDEPENDENT) != 0;
  const cudaError_t e = launch_matvec(a, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)
    return set_error(ASM_E_UNSUPPORTED, "%s: no bulk-copy plan for M=%lld K=%lld", name, (long long)M, (long long)K);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_rowsplit_wait_async(const asm_rowsplit_wait_t* w, void* stream) {
  const char* name = "asm_rowsplit_wait_async";
  if (!w) return set_error(ASM_E_INVALID, "%s: null descriptor", name);
  if (w->n < 0 || w->n > 8) return set_error(ASM_E_INVALID, "%s: n=%d is not in [0, 8]", name, w->n);
  if (w->tp < 1 || w->tp > kMaxTp || w->rank < 0 || w->rank >= w->tp)
    return set_error(ASM_E_INVALID, "%s: tp=%d rank=%d", name, w->tp, w->rank);
  if (w->tp == 1 || w->n == 0) return ASM_OK;  // nothing crosses ranks
  int rc;
  if (!w->seq || !w->done) return set_error(ASM_E_INVALID, "%s: seq and done must be set", name);
  if ((rc = require_device(name, w->seq, "seq")) || (rc = require_device(name, w->done, "done"))) return rc;
  RowsplitWait k;
  k.n = w->n;
  k.tp = w->tp;
  k.rank = w->rank;
  k.seq = w->seq;
  k.done = w->done;
  for (int j = 0; j < w->n; ++j) {
    if (w->M[j] <= 0 || w->M[j] > INT32_MAX / kMaxTp) return set_error(ASM_E_INVALID, "%s: M[%d]=%lld", name, j, (long long)w->M[j]);
    if ((rc = require_device(name, w->own[j], "own")) || (rc = require_device(name, w->y_full[j], "y_full"))) return rc;
    k.own[j] = static_cast<const unsigned long long*>(w->own[j]);
    k.y_full[j] = w->y_full[j];
    k.M[j] = w->M[j];
  }
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const cudaError_t e = launch_rowsplit_wait(k, sms > 0 ? sms : 1, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_matmul_q8q8_async(const int8_t* qweights, const float* scales, const float* x,
                                     float* y, int64_t M, int64_t K, void* stream) {
  return async_matvec("asm_matmul_q8q8_async", kFmtQ8_0, false, false, qweights, scales, x, y,
                      nullptr, M, K, stream);
}

ASMLLM_API int asm_matmul_q8q8_f16s_async(const int8_t* qweights, const uint16_t* scales_f16,
                                          const float* x, float* y, int64_t M, int64_t K,
                                          void* stream) {
  return async_matvec("asm_matmul_q8q8_f16s_async", kFmtQ8_0, false, true, qweights, scales_f16,
                      x, y, nullptr, M, K, stream);
}

ASMLLM_API int asm_matmul_q4_f32_async(const uint8_t* qweights, const float* scales,
                                       const float* x, float* y, int64_t M, int64_t K,
                                       void* stream) {
  return async_matvec("asm_matmul_q4_f32_async", kFmtQ4_0, true, false, qweights, scales, x, y,
                      nullptr, M, K, stream);
}

ASMLLM_API int asm_matmul_q8_async(const int8_t* qweights, const float* scales, const float* x,
                                   float* y, int64_t M, int64_t K, void* stream) {
  return async_matvec("asm_matmul_q8_async", kFmtQ8_0, true, false, qweights, scales, x, y,
                      nullptr, M, K, stream);
}

ASMLLM_API int asm_block_sums_async(int fmt, const void* qweights, const float* scales,
                                    const float* x, float* y, int32_t* isums, int64_t M,
                                    int64_t K, void* stream) {
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0)
    return set_error(ASM_E_INVALID, "asm_block_sums_async: fmt %d is not 2 or 8", fmt);
  if (M > 0 && K > 0 && !isums) return set_error(ASM_E_INVALID, "asm_block_sums_async: isums is NULL");
  return async_matvec("asm_block_sums_async", fmt, false, false, qweights, scales, x, y, isums, M,
                      K, stream);
}

ASMLLM_API int asm_quantize_q8_0_async(const float* x, int8_t* xq, float* xd, int64_t N,
                                       int64_t K, void* stream) {
  const char* name = "asm_quantize_q8_0_async";
  if (N < 0 || K < 0 || K % 32 != 0)
    return set_error(ASM_E_INVALID, "%s: N=%lld K=%lld (K must be a multiple of 32)", name,
                     (long long)N, (long long)K);
  if (N == 0 || K == 0) return ASM_OK;
  int rc;
  if ((rc = require_device(name, x, "x")) || (rc = require_device(name, xq, "xq")) ||
      (rc = require_device(name, xd, "xd")))
    return rc;
  cudaError_t e = launch_quantize(x, xq, xd, N * (K / 32), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int64_t asm_act_image_bytes(int64_t K) {
  if (K < 0 || K % 32 != 0) return -1;
  return (int64_t)act_image_bytes(K / 32);
}

ASMLLM_API int asm_act_image_q8_0_async(const float* x, void* image, int64_t N, int64_t K,
                                        void* stream) {
  const char* name = "asm_act_image_q8_0_async";
  if (N < 0 || K < 0 || K % 32 != 0)
    return set_error(ASM_E_INVALID, "%s: N=%lld K=%lld (K must be a multiple of 32)", name,
                     (long long)N, (long long)K);
  if (N == 0 || K == 0) return ASM_OK;
  int rc;
  if ((rc = require_device(name, x, "x")) || (rc = require_device(name, image, "image"))) return rc;
  if ((uintptr_t)x % 16 != 0 || (uintptr_t)image % 16 != 0)
    return set_error(ASM_E_INVALID, "%s: x and image must be 16-byte aligned", name);
  cudaError_t e = launch_act_image(x, image, N, K, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_act_image_q8_0_prefetch_async(const float* x, void* image, int64_t N, int64_t K,
                                                 const void* next_w, int64_t next_w_bytes,
                                                 const void* next_s, int64_t next_s_bytes,
                                                 void* stream) {
  const char* name = "asm_act_image_q8_0_prefetch_async";
  if (N < 0 || K < 0 || K % 32 != 0 || next_w_bytes < 0 || next_s_bytes < 0)
    return set_error(ASM_E_INVALID, "%s: bad sizes N=%lld K=%lld", name, (long long)N, (long long)K);
  if (N == 0 || K == 0) return ASM_OK;
  int rc;
  if ((rc = require_device(name, x, "x")) || (rc = require_device(name, image, "image"))) return rc;
  if (next_w && next_w_bytes && (rc = require_device(name, next_w, "next_w"))) return rc;
  if (next_s && next_s_bytes && (rc = require_device(name, next_s, "next_s"))) return rc;
  if ((uintptr_t)x % 16 != 0 || (uintptr_t)image % 16 != 0)
    return set_error(ASM_E_INVALID, "%s: x and image must be 16-byte aligned", name);
  cudaError_t e = launch_act_image(x, image, N, K, static_cast<cudaStream_t>(stream), next_w,
                                   (size_t)next_w_bytes, next_s, (size_t)next_s_bytes);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_matmul_image_async(int fmt, const void* qweights, const void* scales,
                                      int scales_are_f16, const void* image, float* y, int64_t M,
                                      int64_t K, void* stream) {
  const char* name = "asm_matmul_image_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0)
    return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  int rc = validate(name, qweights, scales, image, y, M, K);
  if (rc) return rc;
  if (M == 0) return ASM_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if ((rc = check_max_k(name, fmt, false, K, dev))) return rc;
  if ((rc = require_device(name, y, "y"))) return rc;
  if (K > 0) {
    if ((rc = require_device(name, qweights, "qweights")) || (rc = require_device(name, scales, "scales")) ||
        (rc = require_device(name, image, "image")))
      return rc;
    if ((rc = check_align(name, qweights, scales, scales_are_f16 ? 2 : 4, image))) return rc;
  }
  MatvecArgs a;
  a.fmt = fmt;
  a.scales_f16 = scales_are_f16 != 0;
  a.w = qweights;
  a.scales = scales;
  a.image = image;
  a.y = y;
  a.M = M;
  a.K = K;
  a.weights_static = K > 0 && is_static(qweights, weight_bytes(fmt, M, K)) &&
                     is_static(scales, (size_t)M * (K / 32) * (scales_are_f16 ? 2 : 4));
  e = launch_matvec(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_gguf_split_async(int fmt, const uint8_t* raw, uint8_t* qs, void* scales,
                                    int scales_are_f16, int64_t nblocks, void* stream) {
  const char* name = "asm_gguf_split_async";
  if (fmt != kFmtQ4_0 && fmt != kFmtQ8_0)
    return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, fmt);
  if (nblocks < 0) return set_error(ASM_E_INVALID, "%s: negative block count", name);
  if (nblocks == 0) return ASM_OK;
  if ((uintptr_t)raw % 2 != 0 || (uintptr_t)qs % 4 != 0)
    return set_error(ASM_E_INVALID, "%s: raw must be 2-byte and qs 4-byte aligned", name);
  int rc;
  if ((rc = require_device(name, raw, "raw")) || (rc = require_device(name, qs, "qs")) ||
      (rc = require_device(name, scales, "scales")))
    return rc;
  cudaError_t e = launch_gguf_split(fmt, raw, qs, scales, scales_are_f16 ? 1 : 0, nblocks,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_weights_mark_static(const void* ptr, int64_t bytes) {
  if (!ptr || bytes <= 0) return set_error(ASM_E_INVALID, "asm_weights_mark_static: empty range");
  if (classify(ptr, nullptr) != kDevice)
    return set_error(ASM_E_NOT_DEVICE, "asm_weights_mark_static: not a device pointer");
  std::lock_guard<std::mutex> lk(g_static_mu);
  g_static[(uintptr_t)ptr] = (uintptr_t)ptr + (uintptr_t)bytes;
  return ASM_OK;
}

ASMLLM_API int asm_weights_unmark_static(const void* ptr) {
  std::lock_guard<std::mutex> lk(g_static_mu);
  g_static.erase((uintptr_t)ptr);
  return ASM_OK;
}

ASMLLM_API int asm_device_error(unsigned* flags) {
  unsigned v = 0;
  cudaError_t e = read_device_error(&v, true);
  if (e != cudaSuccess) return cuda_error(e, "asm_device_error");
  if (flags) *flags = v;
  return ASM_OK;
}

// Q4_0 x Q8_0 matvec for callers that must not allocate device memory during
// the call (a server that reserves all device memory at start-up, a serving
// loop with a fixed budget, a plugin whose host owns all allocations).  It runs the same two
// kernels as the synchronous path -- the activation-quantize pre-pass into an
// image, then the matvec reading the image -- with the image in the
// library's fixed device array instead of an allocated buffer.  It calls no
// cudaMalloc / cudaFree / allocating routine.  The first call on a device
// looks the array's address up (cudaGetSymbolAddress) and sets up the kernel
// attributes; make that first call before any stream capture.  All calls
// share the one array, so calls that overlap on the GPU (on different streams,
// for instance) race; calls on one stream are ordered.  The array
// keeps the previous call's contents; nothing in it needs clearing, since
// each call rewrites every byte of it that the matvec uses.
ASMLLM_API int asm_matmul_q4_noalloc_async(const uint8_t* qweights, const void* scales,
                                           int scales_are_f16, const float* x, float* y, int64_t M,
                                           int64_t K, void* stream) {
  const char* name = "asm_matmul_q4_noalloc_async";
  int rc = validate(name, qweights, scales, x, y, M, K);
  if (rc) return rc;
  if (K > kNoAllocMaxK)
    return set_error(ASM_E_UNSUPPORTED, "%s: K=%lld exceeds %lld, the size of this entry's fixed scratch", name,
                     (long long)K, (long long)kNoAllocMaxK);
  if (M == 0) return ASM_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return set_error(ASM_E_UNSUPPORTED, "%s: device %d out of range", name, dev);
  if ((rc = require_device(name, y, "y"))) return rc;
  if (K > 0) {
    if ((rc = require_device(name, qweights, "qweights")) || (rc = require_device(name, scales, "scales")) ||
        (rc = require_device(name, x, "x")))
      return rc;
    if ((rc = check_align(name, qweights, scales, scales_are_f16 ? 2 : 4, x))) return rc;
  }
  void* img = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      e = cudaGetSymbolAddress(&g_noalloc_addr[dev], g_noalloc_image);
      if (e != cudaSuccess) {
        g_noalloc_addr[dev] = nullptr;
        return cuda_error(e, "cudaGetSymbolAddress (no-alloc scratch)");
      }
    }
    img = g_noalloc_addr[dev];
  }
  MatvecArgs a;
  a.fmt = kFmtQ4_0;
  a.scales_f16 = scales_are_f16 != 0;
  a.w = qweights;
  a.scales = scales;
  a.image = img;
  a.y = y;
  a.M = M;
  a.K = K;
  a.weights_static = K > 0 && is_static(qweights, weight_bytes(kFmtQ4_0, M, K)) &&
                     is_static(scales, (size_t)M * (K / 32) * (scales_are_f16 ? 2 : 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K > 0) {
    e = launch_act_image(x, img, 1, K, st);
    if (e != cudaSuccess) return cuda_error(e, name);
  }
  e = launch_matvec(a, st);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

// ctypes mirrors of the descriptor (asmllm_b200/native.py FusedMatvec) rely on this layout.
static_assert(sizeof(asm_rows_t) == 80 && offsetof(asm_rows_t, norm_w) == 56 && offsetof(asm_rows_t, tiles) == 72,
              "asm_rows_t layout (asmllm_b200/native.py mirrors it)");
static_assert(sizeof(asm_fused_matvec_t) == 256 && offsetof(asm_fused_matvec_t, eps) == 128 &&
                  offsetof(asm_fused_matvec_t, M) == 144 && offsetof(asm_fused_matvec_t, xchg) == 176,
              "asm_fused_matvec_t layout");

ASMLLM_API int asm_fused_matvec_async(const asm_fused_matvec_t* p, void* stream) {
  const char* name = "asm_fused_matvec_async";
  if (!p) return set_error(ASM_E_INVALID, "%s: null descriptor", name);
  if (p->fmt != kFmtQ4_0 && p->fmt != kFmtQ8_0)
    return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, p->fmt);
  if (p->epilogue < ASM_EPI_STORE || p->epilogue > ASM_EPI_ARGMAX)
    return set_error(ASM_E_INVALID, "%s: unknown epilogue %d", name, p->epilogue);
  if (p->M <= 0 || p->K <= 0 || p->K % 32 != 0 || p->M > INT32_MAX)
    return set_error(ASM_E_INVALID, "%s: need M > 0 and K > 0 a multiple of 32 (M=%lld K=%lld)", name,
                     (long long)p->M, (long long)p->K);
  int rc;
  if ((rc = require_device(name, p->qweights, "qweights")) || (rc = require_device(name, p->scales, "scales")) ||
      (rc = require_device(name, p->y, "y")))
    return rc;
  if ((uintptr_t)p->qweights % 16 || (uintptr_t)p->scales % 16 || (uintptr_t)p->y % 4)
    return set_error(ASM_E_INVALID, "%s: qweights and scales must be 16-byte aligned", name);
  auto dev16 = [&](const void* q, const char* what) -> int {
    if ((rc = require_device(name, q, what))) return rc;
    if ((uintptr_t)q % 16) return set_error(ASM_E_INVALID, "%s: %s must be 16-byte aligned", name, what);
    return ASM_OK;
  };
  if (p->image) {
    if ((rc = dev16(p->image, "image"))) return rc;
    if (p->norm_w || p->embed)
      return set_error(ASM_E_INVALID, "%s: an image prologue takes no norm_w or embed", name);
  } else if (p->embed) {
    if ((rc = dev16(p->embed, "embed")) || (rc = require_device(name, p->tokens, "tokens")) ||
        (rc = require_device(name, p->pos, "pos")))
      return rc;
    if (p->vocab <= 0 || p->max_tokens <= 0)
      return set_error(ASM_E_INVALID, "%s: embed needs vocab > 0 and max_tokens > 0", name);
  } else if ((rc = dev16(p->x, "x"))) {
    return rc;
  }
  if (p->norm_w && (rc = dev16(p->norm_w, "norm_w"))) return rc;
  if (p->x_copy && (rc = dev16(p->x_copy, "x_copy"))) return rc;
  if (p->epilogue == ASM_EPI_SWIGLU) {
    if (p->M % 64 != 0) return set_error(ASM_E_INVALID, "%s: SWIGLU needs M %% 64 == 0 (M=%lld)", name, (long long)p->M);
    if ((rc = dev16(p->h, "h")) || (rc = dev16(p->image_out, "image_out")) ||
        (rc = require_device(name, p->counters, "counters")))
      return rc;
  }
  if (p->epilogue == ASM_EPI_ARGMAX) {
    if ((rc = require_device(name, p->best, "best")) || (rc = require_device(name, p->done, "done")) ||
        (rc = require_device(name, p->tokens, "tokens")) || (rc = require_device(name, p->pos, "pos")))
      return rc;
    if ((uintptr_t)p->best % 8) return set_error(ASM_E_INVALID, "%s: best must be 8-byte aligned", name);
    if (p->max_tokens <= 0) return set_error(ASM_E_INVALID, "%s: ARGMAX needs max_tokens > 0", name);
  }
  MvFuse f;
  f.norm_w = p->norm_w;
  f.eps = p->eps;
  f.embed = p->image ? nullptr : p->embed;
  f.vocab = p->vocab;
  f.tokens = p->tokens;
  f.pos = p->pos;
  f.max_tokens = p->max_tokens;
  f.n_prompt = p->n_prompt;
  f.x_copy = p->x_copy;
  f.h = p->h;
  f.image_out = static_cast<unsigned char*>(p->image_out);
  f.counters = p->counters;
  f.best = reinterpret_cast<unsigned long long*>(p->best);
  f.done = p->done;
  if (p->tp > 1) {
    if (p->tp > kMaxTp || p->tp_rank < 0 || p->tp_rank >= p->tp)
      return set_error(ASM_E_INVALID, "%s: tp %d / rank %d out of range", name, p->tp, p->tp_rank);
    if (p->epilogue != ASM_EPI_RESIDUAL && p->epilogue != ASM_EPI_ARGMAX)
      return set_error(ASM_E_UNSUPPORTED, "%s: tensor parallelism needs the RESIDUAL or ARGMAX epilogue", name);
    if (p->xchg_rows < (p->epilogue == ASM_EPI_RESIDUAL ? p->M : 2))
      return set_error(ASM_E_INVALID, "%s: xchg_rows %d too small", name, p->xchg_rows);
    if ((rc = require_device(name, p->ar_seq, "ar_seq")) || (rc = require_device(name, p->ar_done, "ar_done")))
      return rc;
    for (int r = 0; r < p->tp; ++r) {
      if (!p->xchg[r] || (uintptr_t)p->xchg[r] % 8)
        return set_error(ASM_E_INVALID, "%s: exchange buffer of rank %d missing or misaligned", name, r);
      f.xchg[r] = static_cast<unsigned long long*>(p->xchg[r]);
    }
    f.tp = p->tp;
    f.tp_rank = p->tp_rank;
    f.xchg_rows = p->xchg_rows;
    f.vocab_offset = p->vocab_offset;
    f.ar_seq = p->ar_seq;
    f.ar_done = p->ar_done;
  }
  MatvecArgs a;
  a.fmt = p->fmt;
  a.scales_f16 = true;
  a.w = p->qweights;
  a.scales = p->scales;
  a.x = p->x;
  a.image = p->image;
  a.y = p->y;
  a.M = p->M;
  a.K = p->K;
  a.epi = p->epilogue;
  a.fuse = &f;
  a.weights_static = is_static(p->qweights, weight_bytes(p->fmt, p->M, p->K)) &&
                     is_static(p->scales, (size_t)p->M * (p->K / 32) * 2);
  const cudaError_t e = launch_matvec(a, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)
    return set_error(ASM_E_UNSUPPORTED, "%s: no bulk-copy plan for this shape and fusion (M=%lld K=%lld epilogue %d)",
                     name, (long long)p->M, (long long)p->K, p->epilogue);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_ipc_alloc(int64_t bytes, void** ptr, void* handle64) {
  const char* name = "asm_ipc_alloc";
  if (bytes <= 0 || !ptr || !handle64) return set_error(ASM_E_INVALID, "%s: bad arguments", name);
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return cuda_error(e, name);
  }
  memcpy(handle64, &h, sizeof(h));
  *ptr = p;
  return ASM_OK;
}

ASMLLM_API int asm_ipc_open(const void* handle64, void** ptr) {
  const char* name = "asm_ipc_open";
  if (!handle64 || !ptr) return set_error(ASM_E_INVALID, "%s: bad arguments", name);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_error(e, name);
  *ptr = p;
  return ASM_OK;
}

ASMLLM_API int asm_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? ASM_OK : cuda_error(e, "asm_ipc_close");
}

ASMLLM_API int asm_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? ASM_OK : cuda_error(e, "asm_ipc_free");
}

ASMLLM_API int asm_attention_decode_async(const float* qkv, void* k_cache, void* v_cache,
                                          const float* rope_cs, const int32_t* pos, void* image_out,
                                          int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                          int32_t ctx, float sqrt_head_dim, void* stream) {
  const char* name = "asm_attention_decode_async";
  if (head_dim != 128) return set_error(ASM_E_UNSUPPORTED, "%s: head_dim %d (only 128)", name, head_dim);
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || ctx <= 0)
    return set_error(ASM_E_INVALID, "%s: need n_heads a multiple of n_kv_heads and ctx > 0", name);
  int rc;
  if ((rc = require_device(name, qkv, "qkv")) || (rc = require_device(name, k_cache, "k_cache")) ||
      (rc = require_device(name, v_cache, "v_cache")) || (rc = require_device(name, rope_cs, "rope_cs")) ||
      (rc = require_device(name, pos, "pos")) || (rc = require_device(name, image_out, "image_out")))
    return rc;
  if ((uintptr_t)qkv % 16 || (uintptr_t)k_cache % 16 || (uintptr_t)v_cache % 16 || (uintptr_t)rope_cs % 8 ||
      (uintptr_t)image_out % 16)
    return set_error(ASM_E_INVALID, "%s: misaligned buffer", name);
  const cudaError_t e = launch_attention_decode(qkv, k_cache, v_cache, rope_cs, pos, image_out, n_heads, n_kv_heads,
                                                head_dim, ctx, sqrt_head_dim, static_cast<cudaStream_t>(stream),
                                                g_opt_pdl.load() != 0);
  if (e == cudaErrorNotSupported) return set_error(ASM_E_UNSUPPORTED, "%s: ctx %d too long for shared memory", name, ctx);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

// ---------------------------------------------------------------------------
// Persistent decode (decode_persistent.cu)
// ---------------------------------------------------------------------------
struct DecodeHandle {
  int dev = 0;
  int fmt = 0;
  int sms = 0, per_sm = 0;
  size_t smem = 0;
  int n_ops = 0;
  PersistOp* d_ops = nullptr;
  unsigned* d_sync = nullptr;  // [0] barrier counter, [1] abort word
  unsigned char* d_rep = nullptr;  // replicated x and activation images
  PersistArgs args;
  int ctx = 0, max_tokens = 0;
};

int stage_rows(int fmt, int64_t K) {
  const size_t row_w = (size_t)(K / 32) * (fmt == kFmtQ4_0 ? 16 : 32);
  int R = 8;
  while (R > 2 && (size_t)R * row_w > 16 * 1024) R /= 2;
  return R;
}

// ctypes mirrors (asmllm_b200/native.py DecodeLayer, DecodeModel) rely on these layouts.
static_assert(sizeof(asm_decode_layer_t) == 96, "asm_decode_layer_t layout");
static_assert(sizeof(asm_decode_model_t) == 176 && offsetof(asm_decode_model_t, layers) == 48 &&
                  offsetof(asm_decode_model_t, pos) == 168,
              "asm_decode_model_t layout");

ASMLLM_API int asm_decode_create(const asm_decode_model_t* m, void** handle) {
  const char* name = "asm_decode_create";
  if (!m || !handle) return set_error(ASM_E_INVALID, "%s: null argument", name);
  *handle = nullptr;
  if (m->fmt != kFmtQ4_0 && m->fmt != kFmtQ8_0) return set_error(ASM_E_INVALID, "%s: fmt %d is not 2 or 8", name, m->fmt);
  if (m->head_dim != 128) return set_error(ASM_E_UNSUPPORTED, "%s: head_dim %d (only 128)", name, m->head_dim);
  if (m->n_layers <= 0 || m->n_heads <= 0 || m->n_kv_heads <= 0 || m->n_heads % m->n_kv_heads || m->vocab <= 0 ||
      m->ctx <= 0 || m->max_tokens <= 1 || !m->layers)
    return set_error(ASM_E_INVALID, "%s: bad model dimensions", name);
  const int64_t qdim = (int64_t)m->n_heads * m->head_dim;
  if (m->dim % 256 || m->ffn % 256 || qdim % 256)
    return set_error(ASM_E_UNSUPPORTED, "%s: dim, ffn and n_heads*head_dim must be multiples of 256", name);
  int rc;
  auto dev16 = [&](const void* q, const char* what) -> int {
    if ((rc = require_device(name, q, what))) return rc;
    if ((uintptr_t)q % 16) return set_error(ASM_E_INVALID, "%s: %s must be 16-byte aligned", name, what);
    return ASM_OK;
  };
  for (int l = 0; l < m->n_layers; ++l) {
    const asm_decode_layer_t& L = m->layers[l];
    const void* ptrs[] = {L.wqkv, L.sqkv, L.wo, L.so, L.wgu, L.sgu, L.wdown, L.sdown, L.attn_norm, L.ffn_norm, L.k_cache, L.v_cache};
    for (const void* q : ptrs)
      if ((rc = dev16(q, "a layer buffer"))) return rc;
  }
  const void* globals[] = {m->lm_head, m->lm_scales, m->final_norm, m->embed, m->rope_cs, m->x, m->qkv, m->img_attn,
                           m->h, m->img_h, m->counters, m->logits, m->best, m->tokens, m->pos};
  for (const void* q : globals)
    if ((rc = dev16(q, "a model buffer"))) return rc;

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  int sms = 0, optin = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);

  // Replicated activations of the persistent kernel: x [xr][dim], then the
  // two images [xr][bytes] (each replica 16-byte aligned).
  const int xr = 1;  // measured: 8 replicas were no faster than 1 on B200
  const size_t x_bytes = (size_t)m->dim * sizeof(float);
  const size_t ia_bytes = act_image_bytes(qdim / 32), ih_bytes = act_image_bytes(m->ffn / 32);
  unsigned char* d_rep = nullptr;
  e = cudaMalloc(&d_rep, (size_t)xr * (x_bytes + ia_bytes + ih_bytes));
  if (e != cudaSuccess) return cuda_error(e, name);
  float* x_rep = reinterpret_cast<float*>(d_rep);
  unsigned char* ia_rep = d_rep + (size_t)xr * x_bytes;
  unsigned char* ih_rep = ia_rep + (size_t)xr * ia_bytes;

  std::vector<PersistOp> ops;
  auto mv = [&](const void* w, const void* sc, int M, int64_t K, int pro, int epi) {
    PersistOp o;
    o.kind = kOpMatvec;
    o.pro = pro;
    o.epi = epi;
    o.M = M;
    o.nb = (int)(K / 32);
    o.R = stage_rows(m->fmt, K);
    o.w = static_cast<const uint8_t*>(w);
    o.s = static_cast<const __half*>(sc);
    return o;
  };
  const int qkv_rows = (m->n_heads + 2 * m->n_kv_heads) * m->head_dim;
  for (int l = 0; l < m->n_layers; ++l) {
    const asm_decode_layer_t& L = m->layers[l];
    PersistOp o = mv(L.wqkv, L.sqkv, qkv_rows, m->dim, kProNorm, kEpiStore);
    o.from_embed = l == 0;
    o.x = x_rep;
    o.norm_w = L.attn_norm;
    o.y = m->qkv;
    ops.push_back(o);
    PersistOp at;
    at.kind = kOpAttention;
    at.first_of_step = l == 0;
    at.kc = static_cast<__half*>(L.k_cache);
    at.vc = static_cast<__half*>(L.v_cache);
    ops.push_back(at);
    o = mv(L.wo, L.so, m->dim, qdim, kProImage, kEpiResidual);
    o.image = ia_rep;
    o.image_stride = ia_bytes;
    o.y = x_rep;
    ops.push_back(o);
    o = mv(L.wgu, L.sgu, 2 * m->ffn, m->dim, kProNorm, kEpiSwiglu);
    o.x = x_rep;
    o.norm_w = L.ffn_norm;
    ops.push_back(o);
    o = mv(L.wdown, L.sdown, m->dim, m->ffn, kProImage, kEpiResidual);
    o.image = ih_rep;
    o.image_stride = ih_bytes;
    o.y = x_rep;
    ops.push_back(o);
  }
  PersistOp lm = mv(m->lm_head, m->lm_scales, m->vocab, m->dim, kProNorm, kEpiArgmax);
  lm.x = x_rep;
  lm.norm_w = m->final_norm;
  lm.y = m->logits;
  ops.push_back(lm);

  DecodeHandle* hd = new DecodeHandle();
  hd->dev = dev;
  hd->fmt = m->fmt;
  hd->sms = sms;
  hd->n_ops = (int)ops.size();
  hd->ctx = m->ctx;
  hd->max_tokens = m->max_tokens;
  PersistArgs& a = hd->args;
  a.n_ops = hd->n_ops;
  a.eps = m->eps;
  a.sqrt_hd = m->sqrt_head_dim;
  a.embed = m->embed;
  a.vocab = m->vocab;
  a.rope = reinterpret_cast<const float2*>(m->rope_cs);
  a.ctx = m->ctx;
  a.n_heads = m->n_heads;
  a.n_kv = m->n_kv_heads;
  a.xr = xr;
  a.x_stride = (size_t)m->dim;
  a.img_attn_stride = ia_bytes;
  a.img_h_stride = ih_bytes;
  a.x = x_rep;
  a.qkv = m->qkv;
  a.img_attn = ia_rep;
  a.h = m->h;
  a.img_h = ih_rep;
  hd->d_rep = d_rep;
  a.counters = m->counters;
  a.best = reinterpret_cast<unsigned long long*>(m->best);
  a.tokens = m->tokens;
  a.pos = m->pos;
  a.max_tokens = m->max_tokens;
  a.err = device_error_word();
  if (!persist_plan(a, ops, m->fmt, optin, &hd->per_sm, &hd->smem)) {
    cudaFree(d_rep);
    delete hd;
    return set_error(ASM_E_UNSUPPORTED, "%s: no shared-memory plan for these widths", name);
  }
  if (!a.err) {
    cudaFree(d_rep);
    delete hd;
    return set_error(ASM_E_CUDA, "%s: device error word unavailable", name);
  }
  e = cudaMalloc(&hd->d_ops, ops.size() * sizeof(PersistOp));
  if (e == cudaSuccess) e = cudaMalloc(&hd->d_sync, 2 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemcpy(hd->d_ops, ops.data(), ops.size() * sizeof(PersistOp), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(hd->d_ops);
    cudaFree(hd->d_sync);
    cudaFree(d_rep);
    delete hd;
    return cuda_error(e, name);
  }
  a.ops = hd->d_ops;
  a.sync = hd->d_sync;
  a.abort = hd->d_sync + 1;
  *handle = hd;
  return ASM_OK;
}

ASMLLM_API int asm_decode_run_async(void* handle, int32_t n_steps, int32_t n_prompt, void* stream) {
  const char* name = "asm_decode_run_async";
  DecodeHandle* hd = static_cast<DecodeHandle*>(handle);
  if (!hd) return set_error(ASM_E_INVALID, "%s: null handle", name);
  if (n_steps <= 0 || n_steps > hd->ctx || n_prompt < 0)
    return set_error(ASM_E_INVALID, "%s: need 0 < n_steps <= ctx and n_prompt >= 0", name);
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != hd->dev) return set_error(ASM_E_INVALID, "%s: handle belongs to device %d, current is %d", name, hd->dev, cur);
  PersistArgs a = hd->args;
  a.n_steps = n_steps;
  a.n_prompt = n_prompt;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(hd->d_sync, 0, 2 * sizeof(unsigned), st);
  if (e == cudaSuccess) e = launch_decode_persistent(a, hd->fmt, hd->smem, hd->sms, hd->per_sm, st);
  if (e != cudaSuccess) return cuda_error(e, name);
  return ASM_OK;
}

ASMLLM_API int asm_decode_destroy(void* handle) {
  DecodeHandle* hd = static_cast<DecodeHandle*>(handle);
  if (!hd) return ASM_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(hd->dev);
  cudaFree(hd->d_ops);
  cudaFree(hd->d_sync);
  cudaFree(hd->d_rep);
  cudaSetDevice(cur);
  delete hd;
  return ASM_OK;
}

ASMLLM_API int asm_set_option(const char* name, int value) {
  if (!name) return -1;
  if (strcmp(name, "tma") == 0) return g_opt_tma.exchange(value ? 1 : 0);
  if (strcmp(name, "pdl") == 0) return g_opt_pdl.exchange(value ? 1 : 0);
  if (strcmp(name, "gemm_splits") == 0) return g_opt_gemm_splits.exchange(value < 0 ? 0 : value);
  if (strcmp(name, "image_min_k") == 0) return g_opt_image_min_k.exchange(value < 0 ? 0 : value);
  if (strcmp(name, "sync_map") == 0) return g_opt_sync_map.exchange(value & 3);
  if (strcmp(name, "mv_rows") == 0) return g_opt_mv_rows.exchange(value == 1 || value == 2 || value == 4 ? value : 0);
  if (strcmp(name, "mv_slots") == 0) return g_opt_mv_slots.exchange(value < 0 ? 0 : value);
  if (strcmp(name, "mv_smem_kb") == 0) return g_opt_mv_smem_kb.exchange(value <= 0 ? 0 : value < 16 ? 16 : value);
  if (strcmp(name, "mv_ctas") == 0) return g_opt_mv_ctas.exchange(value < 1 ? 1 : value > 4 ? 4 : value);
  if (strcmp(name, "sync_fused") == 0) return g_opt_sync_fused.exchange(value ? 1 : 0);
  if (strcmp(name, "image_prefetch_mb") == 0)
    return g_opt_image_prefetch_mb.exchange(value < 0 ? 0 : value > 4096 ? 4096 : value);
  if (strcmp(name, "mv_kernel") == 0) return g_opt_mv_kernel.exchange(value == 1 || value == 2 ? value : 0);
  if (strcmp(name, "xchg_wait_us") == 0) {
    // SM clock cycles at about 2 GHz; set on the current device
    const int v = value < 0 ? 0 : value;
    const cudaError_t e = set_xchg_wait_cycles(v > 0 ? (long long)v * 2000LL : 0LL);
    if (e != cudaSuccess) {
      cuda_error(e, "asm_set_option(xchg_wait_us)");
      return -1;
    }
    return g_opt_xchg_wait_us.exchange(v);
  }
  set_error(ASM_E_INVALID, "asm_set_option: unknown option '%s'", name);
  return -1;
}

ASMLLM_API int64_t asm_max_k(int fmt, int fp32_activations) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return max_k(fmt == kFmtQ8_0 ? kFmtQ8_0 : kFmtQ4_0, fp32_activations != 0, dev);
}

ASMLLM_API const char* asm_version(void) { return "asmllm-b200 0.1 (sm_100a)"; }

}  // extern "C"
