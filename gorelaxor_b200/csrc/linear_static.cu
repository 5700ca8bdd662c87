// grx_linear_q8_static: kern.Linear's int8 path with no allocation, for
// hosts that cannot call cudaMalloc (their pool allocator owns the device's
// memory, or a real-time loop must not stall the device). The rounded
// activations, the only scratch the int8 path needs, live in one fixed
// array of this file; the caller passes device inputs and outputs.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/grx.h"
#include "kernels.h"

namespace grx {
int set_error(int code, const char* msg);
int weight_device(const grx_weight* w);
bool weight_q8(const grx_weight* w, const DQ8** q8, bool* dropped);
}  // namespace grx

using namespace grx;

namespace {

// int8 activations [m][cols], then their (s, s) block scales from a 256-byte
// boundary: at most GRX_STATIC_MAX_ELEMS + GRX_STATIC_MAX_ELEMS / 32 * 8.
constexpr size_t kScratchBytes = size_t(GRX_STATIC_MAX_ELEMS) + size_t(GRX_STATIC_MAX_ELEMS) / 32 * 8;

// Host code sees only a stand-in under this name; the device address comes
// from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) uint8_t g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// The array's address on `dev`, which must be the current device.
int scratch_on(int dev, uint8_t** out) {
  if (dev < 0 || dev >= kMaxDevices) return set_error(GRX_ENODEV, "grx_linear_q8_static: device out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess)
      return set_error(GRX_ECUDA, (std::string("grx_linear_q8_static: cudaGetSymbolAddress: ") +
                                   cudaGetErrorString(e)).c_str());
    g_addr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_addr[dev]);
  return GRX_OK;
}

// Puts the caller's current device back on every return path: the hosts this
// entry point serves own their device state.
struct DeviceGuard {
  int prev = -1;
  DeviceGuard() {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int grx_linear_q8_static(const grx_weight* w, const float* d_x, int m, const float* d_bias,
                                    float* d_dst, void* stream) {
  if (!w || !d_x || !d_dst || m < 0) return set_error(GRX_EINVAL, "grx_linear_q8_static: bad argument");
  const DQ8* q8 = nullptr;
  bool dropped = false;
  if (!weight_q8(w, &q8, &dropped)) return set_error(GRX_EINVAL, "grx_linear_q8_static: the weight is not Q8_0");
  if (!dropped && m < 2)
    return set_error(GRX_EINVAL, "grx_linear_q8_static: one row on a weight with rows kept takes the float path; "
                                 "use grx_linear");
  if (m == 0) return GRX_OK;
  const int n = q8->rows, k = q8->cols;
  if (m > 8 && k % 64 != 0)
    return set_error(GRX_EINVAL, "grx_linear_q8_static: int8 products of more than 8 rows need K % 64 == 0");
  if (m <= 8 && n % 32 != 0)
    return set_error(GRX_EINVAL, "grx_linear_q8_static: int8 products of up to 8 rows need N % 32 == 0");
  const size_t elems = size_t(m) * size_t(k);
  if (elems > size_t(GRX_STATIC_MAX_ELEMS))
    return set_error(GRX_ERANGE, ("grx_linear_q8_static: m*cols = " + std::to_string(elems) +
                                  " is above the fixed scratch of " + std::to_string(GRX_STATIC_MAX_ELEMS) +
                                  " values; split the rows or use grx_linear")
                                     .c_str());
  const int dev = weight_device(w);
  const DeviceGuard keep;
  cudaError_t e = cudaSetDevice(dev);
  if (e != cudaSuccess)
    return set_error(GRX_ECUDA, (std::string("grx_linear_q8_static: cudaSetDevice: ") + cudaGetErrorString(e)).c_str());
  uint8_t* base = nullptr;
  const int rc = scratch_on(dev, &base);
  if (rc) return rc;
  int8_t* q = reinterpret_cast<int8_t*>(base);
  float2* s = reinterpret_cast<float2*>(base + (elems + 255) / 256 * 256);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch_quant(d_x, m, k, q, s, st);
  EpiArgs ep;
  ep.epi = EPI_STORE;
  ep.y = d_dst;
  ep.ldy = n;
  ep.bias = d_bias;
  launch_q8_product(q, s, m, *q8, ep, st);
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(GRX_ECUDA, (std::string("grx_linear_q8_static: launch: ") + cudaGetErrorString(e)).c_str());
  return GRX_OK;
}
