// Allocation-free BlockSparse encoder entry point.
//
// This entry point has no counterpart in the reference: it exists for callers
// of this library that cannot allocate device memory themselves — code running
// under a custom allocator or memory pool that forbids cudaMalloc, plugins whose
// host application owns all device memory, or paths that must not touch the
// allocator (and so cannot hand us a scratch buffer).  It encodes exactly like
// the regular BlockSparse encoder (same kernel, same bytes) but keeps the
// encoder's scratch in a fixed, file-scope device array instead of asking for
// a scratch buffer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest number of int16 codes one call accepts (64 Mi).  The scratch array
// behind it holds one look-back status word per tile of 16384 codes (4096
// tiles at the limit), a tile counter and a few spare words: 4104 u64, about
// 32 KiB, which every GPU that loads this library keeps until exit.
int64_t ngl_bs_encode_noalloc_max_n(void);

// Encode `n` int16 error-bounded codes into the BlockSparse byte stream
// ([u32 n] then per 32-code block [u32 mask][i16 per non-zero]) on `stream`.
//   codes        device pointer, n int16 values
//   out          device pointer, capacity of at least 4 + 68 * ceil(n / 32) bytes
//   total_bytes  device pointer to one uint64: receives the stream length
//   status       device pointer to int32[4]; each call clears it on `stream`
//                before its kernel runs, then the kernel records the first
//                error it meets (it never traps).  After the stream has
//                finished, status[0] is
//                  0  success
//                  4  an output or scratch bound was exceeded
//                  6  a look-back wait on a predecessor tile gave up after
//                     2 s (the stream is then incomplete)
//                and status[1] holds the tile concerned.
// Returns 0 (cudaSuccess) when the work was enqueued, the CUDA error code of a
// failed set-up or launch, or -2 when n exceeds ngl_bs_encode_noalloc_max_n().
//
// The first call on a device looks up the scratch array's device address
// (cudaGetSymbolAddress, with that device current) and keeps it for the
// process; make that first call before any stream capture.  cudaDeviceReset
// after that first call is not supported: it unloads the module, and the
// kept address would be stale.  No call allocates or frees memory.  All calls
// share the one scratch array, which keeps the last call's contents (each call
// clears the part it needs before its kernel runs); calls that overlap on the
// GPU, e.g. on two streams at once, race on it and must be serialised by the
// caller.
int ngl_bs_encode_noalloc(const int16_t* codes, int64_t n, uint8_t* out, uint64_t* total_bytes, int* status,
                          cudaStream_t stream);

// Text for a return code of ngl_bs_encode_noalloc.
const char* ngl_bs_encode_noalloc_error(int code);

#ifdef __cplusplus
}
#endif
