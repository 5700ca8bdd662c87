// Host-side helpers shared by the C-ABI files (see host.h).
#include "host.h"

#include <cstring>
#include <mutex>

#include "gguf.h"

namespace grx {
void q8_kernels_init();

namespace {
thread_local std::string g_err;
}

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

const std::string& last_error_message() { return g_err; }

// Device setup done once per device: kernel attributes.
int device_init(int dev) {
  static std::mutex mu;
  static std::vector<bool> done(64, false);
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || dev < 0 || dev >= n || dev >= 64)
    return fail(GRX_ENODEV, "no CUDA device " + std::to_string(dev));
  CK(cudaSetDevice(dev));
  std::lock_guard<std::mutex> lk(mu);
  if (!done[size_t(dev)]) {
    q8_kernels_init();
    flow_kernels_init();
    tdt_kernels_init();
    whisper_kernels_init();
    mimi_kernels_init();
    attn_kernels_init();
    fconf_kernels_init();
    cudaError_t e = cudaGetLastError();  // attribute calls report here; clear it
    if (e != cudaSuccess) return fail(GRX_ECUDA, std::string("kernel attributes: ") + cudaGetErrorString(e));
    done[size_t(dev)] = true;
  }
  return GRX_OK;
}

// Splits rows×cols Q8_0 blocks (34 bytes: f16 scale, 32 int8) into the
// device layout: int8 values [rows][cols] and f16 scales [rows][cols/32].
DQ8 upload_q8(Arena& ar, const uint8_t* blocks, int rows, int cols, int* rc) {
  DQ8 w;
  w.rows = rows;
  w.cols = cols;
  size_t nb = size_t(cols) / 32;
  std::vector<int8_t> q(size_t(rows) * cols);
  std::vector<uint16_t> d(size_t(rows) * nb);
  for (size_t b = 0; b < size_t(rows) * nb; b++) {
    const uint8_t* blk = blocks + b * 34;
    d[b] = uint16_t(blk[0] | blk[1] << 8);
    std::memcpy(&q[b * 32], blk + 2, 32);
  }
  // dw and -1.5·2^23·dw, block-major: the product is exact in float32 for
  // every finite half (at most 12 significant bits, far from over- or
  // underflow).
  std::vector<float> dwT(d.size()), nmT(d.size());
  for (size_t r = 0; r < size_t(rows); r++)
    for (size_t b = 0; b < nb; b++) {
      float dw = f16_to_f32(d[r * nb + b]);
      dwT[b * rows + r] = dw;
      nmT[b * rows + r] = -12582912.0f * dw;
    }
  w.q = ar.upload(q.data(), q.size(), rc);
  w.d = ar.upload(d.data(), d.size(), rc);
  const size_t np = (size_t(rows) + 1) / 2;
  std::vector<float> quads(nb * np * 4, 0.f);
  for (size_t b = 0; b < nb; b++)
    for (size_t r = 0; r < size_t(rows); r++) {
      float* q4 = &quads[(b * np + r / 2) * 4];
      q4[r & 1] = dwT[b * rows + r];
      q4[2 + (r & 1)] = nmT[b * rows + r];
    }
  w.dwnm = reinterpret_cast<const float4*>(ar.upload(quads.data(), quads.size(), rc));
  return w;
}

}  // namespace grx
