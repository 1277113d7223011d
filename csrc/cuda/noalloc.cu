// Allocation-free BlockSparse encoder (declared in noalloc.h; it has no
// counterpart in the reference).  The look-back scratch of the encoder lives
// in a file-scope device array; host code passes its device address, looked
// up once per device with cudaGetSymbolAddress.
#include <mutex>

#include "codecs.h"
#include "noalloc.h"

namespace {

constexpr int64_t kMaxN = int64_t(1) << 26;  // 64 Mi codes
// One status word per tile of kPackTileBlocks * 32 = 16384 codes (4096 tiles
// at kMaxN), the tile counter and spare words: 4104 u64 = 32,832 bytes.
constexpr int64_t kScratchWords =
    ((kMaxN + 31) / 32 + ngl::codec::kPackTileBlocks - 1) / ngl::codec::kPackTileBlocks + 8;
static_assert(kScratchWords == 4104, "scratch size documented in noalloc.h");

// The scratch itself.  In host code `g_scratch` only names a host-side stand-in
// for the symbol, never a device address: kernels get the address from
// cudaGetSymbolAddress below.
static __device__ __align__(256) uint64_t g_scratch[kScratchWords];

constexpr int kMaxDevices = 64;
uint64_t* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

// Once per device, with that device current.
cudaError_t scratch_for_current_device(uint64_t** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<uint64_t*>(p);
  }
  *ptr = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int64_t ngl_bs_encode_noalloc_max_n(void) { return kMaxN; }

extern "C" int ngl_bs_encode_noalloc(const int16_t* codes, int64_t n, uint8_t* out, uint64_t* total_bytes,
                                     int* status, cudaStream_t stream) {
  if (n < 0 || n > kMaxN) return -2;
  if (ngl::codec::pack_scratch_words(n) > kScratchWords) return -2;
  uint64_t* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return (int)e;
  // The kernel only records errors (first one wins), so the success value
  // comes from clearing the caller's status words here.  Allocates nothing.
  if (status != nullptr) {
    e = cudaMemsetAsync(status, 0, 4 * sizeof(int), stream);
    if (e != cudaSuccess) return (int)e;
  }
  // The encoder clears the scratch words it uses (cudaMemsetAsync) before its
  // kernel runs, so the previous call's contents do not leak into this one.
  e = ngl::codec::bs_encode(codes, n, out, scratch, total_bytes, status, stream);
  return (int)e;
}

extern "C" const char* ngl_bs_encode_noalloc_error(int code) {
  if (code == 0) return "success";
  if (code == -2) return "n exceeds ngl_bs_encode_noalloc_max_n() (67108864 codes)";
  return cudaGetErrorString((cudaError_t)code);
}
