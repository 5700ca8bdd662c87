// Host-side helpers shared by the files that implement the C ABI: the
// per-thread error message, the one-time set-up of a device, device
// allocations freed together, and the Q8_0 upload.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/grx.h"
#include "kernels.h"

namespace grx {

// Records msg as the calling thread's last error and returns code.
int fail(int code, const std::string& msg);
const std::string& last_error_message();

// Once per device: kernel attributes (dynamic shared memory opt-ins).
int device_init(int dev);

// Device allocations of one owner, freed together on its device.
struct Arena {
  int dev = 0;
  std::vector<void*> ptrs;
  size_t bytes = 0;
  template <class T>
  T* alloc(size_t n, int* rc) {
    void* p = nullptr;
    if (*rc) return nullptr;
    if (n == 0) n = 1;
    cudaError_t e = cudaMalloc(&p, n * sizeof(T));
    if (e != cudaSuccess) {
      *rc = fail(GRX_ENOMEM, "cudaMalloc of " + std::to_string(n * sizeof(T)) + " bytes: " + cudaGetErrorString(e));
      return nullptr;
    }
    ptrs.push_back(p);
    bytes += n * sizeof(T);
    return (T*)p;
  }
  template <class T>
  T* upload(const T* h, size_t n, int* rc) {
    T* p = alloc<T>(n, rc);
    if (p && cudaMemcpy(p, h, n * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess)
      *rc = fail(GRX_ECUDA, "upload failed");
    return p;
  }
  Arena() = default;
  Arena(const Arena&) = delete;
  Arena& operator=(const Arena&) = delete;
  ~Arena() {
    if (ptrs.empty()) return;
    cudaSetDevice(dev);
    for (void* p : ptrs) cudaFree(p);
  }
};

// Splits rows×cols Q8_0 blocks (34 bytes: f16 scale, 32 int8) into the
// device layout of DQ8.
DQ8 upload_q8(Arena& ar, const uint8_t* blocks, int rows, int cols, int* rc);

}  // namespace grx

#define CK(call)                                                                                    \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess) return fail(GRX_ECUDA, std::string(#call ": ") + cudaGetErrorString(e_)); \
  } while (0)
