// abi.cu -- error reporting, version query, and the two stream-less utility kernels of the
// C ABI: Q4_K dequant (config 1) and the seeded synthetic block generator.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace b2host {
static thread_local char g_err[512] = "";

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char *what) {
  return set_error(B200MOE_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}
}  // namespace b2host

using namespace b2;

// --------------------------------------------------------------------------------- dequant
// One thread per 16-byte quant chunk (8 threads per super-block). Each thread reads the
// block header (16 B, shared by the 8 threads of its block) and its chunk, and writes 32
// values: two runs of 16 consecutive elements. Value = fmaf(d*sc, q, -(dmin*m)): the
// products are exact, so this is the single rounding of the reference's f64 expression
// (tools/gguf_reader.py:248-267 / tools/gguf_fast_dequant.py:109-125).
template <bool kBF16>
__global__ void __launch_bounds__(256) k_q4k_dequant(const uint8_t *__restrict__ blocks, int64_t nblocks,
                                                     void *__restrict__ out) {
  const int64_t nthreads = nblocks * 8;
  for (int64_t tid = (int64_t)blockIdx.x * 256 + threadIdx.x; tid < nthreads;
       tid += (int64_t)gridDim.x * 256) {
    const int64_t b = tid >> 3;
    const int c = (int)(tid & 7);
    const uint8_t *blk = blocks + b * kQB;
    const uint4 h = ldg_stream(blk);
    const uint4 q = ldg_stream(blk + 16 + 16 * c);
    float s0, m0, s1, m1;
    q4k_scales(h, c, s0, m0, s1, m1);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    float lo[16], hi[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t ml = w[i] & 0x0F0F0F0Fu, mh = (w[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        lo[4 * i + k] = __fmaf_rn(s0, nib_f(ml, k), -m0);
        hi[4 * i + k] = __fmaf_rn(s1, nib_f(mh, k), -m1);
      }
    }
    const int64_t e0 = b * 256 + chunk_pos(0, c);
    if (kBF16) {
      uint16_t *o = reinterpret_cast<uint16_t *>(out) + e0;
      uint32_t pl[8], ph[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        pl[i] = (uint32_t)f2bf(lo[2 * i]) | ((uint32_t)f2bf(lo[2 * i + 1]) << 16);
        ph[i] = (uint32_t)f2bf(hi[2 * i]) | ((uint32_t)f2bf(hi[2 * i + 1]) << 16);
      }
      __stcs(reinterpret_cast<uint4 *>(o), make_uint4(pl[0], pl[1], pl[2], pl[3]));
      __stcs(reinterpret_cast<uint4 *>(o + 8), make_uint4(pl[4], pl[5], pl[6], pl[7]));
      __stcs(reinterpret_cast<uint4 *>(o + 32), make_uint4(ph[0], ph[1], ph[2], ph[3]));
      __stcs(reinterpret_cast<uint4 *>(o + 40), make_uint4(ph[4], ph[5], ph[6], ph[7]));
    } else {
      float *o = reinterpret_cast<float *>(out) + e0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __stcs(reinterpret_cast<float4 *>(o + 4 * i), make_float4(lo[4 * i], lo[4 * i + 1], lo[4 * i + 2], lo[4 * i + 3]));
        __stcs(reinterpret_cast<float4 *>(o + 32 + 4 * i),
               make_float4(hi[4 * i], hi[4 * i + 1], hi[4 * i + 2], hi[4 * i + 3]));
      }
    }
  }
}

// --------------------------------------------------------------------------------- synth
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {  // splitmix64 output function
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// One thread per block; the field law and word map are documented at
// oracle/q4k.py synth_blocks, which is this kernel's host mirror.
__global__ void __launch_bounds__(256) k_synth_q4k(uint64_t key, int64_t block0, int64_t nblocks,
                                                   uint8_t *__restrict__ out) {
  for (int64_t b = (int64_t)blockIdx.x * 256 + threadIdx.x; b < nblocks; b += (int64_t)gridDim.x * 256) {
    const uint64_t base = (uint64_t)(block0 + b) * 19ull;
    uint64_t w[19];
#pragma unroll
    for (int i = 0; i < 19; ++i) w[i] = mix64(key + kGolden * (base + (uint64_t)i + 1ull));
    const float ud = (float)(uint32_t)(w[0] & 0xFFFFFFull) * 5.9604644775390625e-8f;
    const float um = (float)(uint32_t)((w[0] >> 32) & 0xFFFFFFull) * 5.9604644775390625e-8f;
    const float d32 = __fadd_rn(1e-3f, __fmul_rn(ud, 9e-3f));
    const float m32 = __fmul_rn(um, 5e-3f);
    const uint32_t dh = __half_as_ushort(__float2half_rn(d32));
    const uint32_t mh = __half_as_ushort(__float2half_rn(m32));
    uint4 *o = reinterpret_cast<uint4 *>(out + b * kQB);
    o[0] = make_uint4(dh | (mh << 16), (uint32_t)w[1], (uint32_t)(w[1] >> 32), (uint32_t)w[2]);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o[1 + i] = make_uint4((uint32_t)w[3 + 2 * i], (uint32_t)(w[3 + 2 * i] >> 32), (uint32_t)w[4 + 2 * i],
                            (uint32_t)(w[4 + 2 * i] >> 32));
  }
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

extern "C" {

int b200moe_abi_version(void) { return B200MOE_ABI_VERSION; }

const char *b200moe_last_error(void) { return b2host::g_err; }

int b200moe_q4k_dequant(const void *blocks, int64_t nblocks, void *out, int out_dtype, void *stream) {
  if (nblocks < 0) return b2host::set_error(B200MOE_EINVAL, "q4k_dequant: nblocks=%lld < 0", (long long)nblocks);
  if (nblocks == 0) return B200MOE_OK;
  if (!blocks || !out) return b2host::set_error(B200MOE_EINVAL, "q4k_dequant: NULL pointer");
  if (!aligned16(blocks) || !aligned16(out))
    return b2host::set_error(B200MOE_EINVAL, "q4k_dequant: pointers must be 16-byte aligned");
  if (out_dtype != B200MOE_F32 && out_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "q4k_dequant: out_dtype %d is neither F32 nor BF16", out_dtype);
  const int64_t threads = nblocks * 8;
  int64_t grid = (threads + 255) / 256;
  if (grid > 148 * 64) grid = 148 * 64;
  cudaStream_t s = (cudaStream_t)stream;
  if (out_dtype == B200MOE_BF16)
    k_q4k_dequant<true><<<(unsigned)grid, 256, 0, s>>>((const uint8_t *)blocks, nblocks, out);
  else
    k_q4k_dequant<false><<<(unsigned)grid, 256, 0, s>>>((const uint8_t *)blocks, nblocks, out);
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

int b200moe_synth_q4k(uint64_t seed, uint32_t stream_id, int64_t block0, int64_t nblocks, void *out,
                      void *stream) {
  if (nblocks < 0 || block0 < 0)
    return b2host::set_error(B200MOE_EINVAL, "synth_q4k: negative block range");
  if (nblocks == 0) return B200MOE_OK;
  if (!out || !aligned16(out)) return b2host::set_error(B200MOE_EINVAL, "synth_q4k: out NULL or unaligned");
  const uint64_t key = mix64(seed + kGolden * ((uint64_t)stream_id + 1ull));
  int64_t grid = (nblocks + 255) / 256;
  if (grid > 148 * 64) grid = 148 * 64;
  k_synth_q4k<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(key, block0, nblocks, (uint8_t *)out);
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

}  // extern "C"

// --------------------------------------------------------------------------------- peer memory
// CUDA IPC for the peer-memory form of expert parallelism: a rank exports the allocation that
// holds one of its buffers and the other ranks (other processes, other GPUs of the node) map it,
// after which their kernels store into it over NVLink. Legacy IPC maps plain device memory:
// no multicast object is created.
#include <cuda.h>
#include <string.h>

namespace {
using AddrRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

int alloc_base(const void *p, void **base) {
  static AddrRangeFn fn = nullptr;
  if (!fn) {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    B2_CUDA(cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !f)
      return b2host::set_error(B200MOE_ECUDA, "cuMemGetAddressRange is not available from the driver");
    fn = (AddrRangeFn)f;
  }
  CUdeviceptr b = 0;
  size_t n = 0;
  const CUresult r = fn(&b, &n, (CUdeviceptr)p);
  if (r != CUDA_SUCCESS) return b2host::set_error(B200MOE_EINVAL, "ipc: %p is not device memory (%d)", p, (int)r);
  *base = (void *)b;
  return B200MOE_OK;
}
}  // namespace

extern "C" {

int b200moe_ipc_handle(const void *dptr, void *handle, int64_t *offset) {
  if (!dptr || !handle || !offset) return b2host::set_error(B200MOE_EINVAL, "ipc_handle: NULL argument");
  void *base = nullptr;
  int rc = alloc_base(dptr, &base);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  B2_CUDA(cudaIpcGetMemHandle(&h, base));
  static_assert(sizeof(h) == B200MOE_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)((const char *)dptr - (const char *)base);
  return B200MOE_OK;
}

int b200moe_ipc_open(const void *handle, int64_t offset, void **dptr) {
  if (!handle || !dptr || offset < 0) return b2host::set_error(B200MOE_EINVAL, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  B2_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *dptr = (char *)base + offset;
  return B200MOE_OK;
}

int b200moe_ipc_close(void *dptr, int64_t offset) {
  if (!dptr) return B200MOE_OK;
  B2_CUDA(cudaIpcCloseMemHandle((char *)dptr - offset));
  return B200MOE_OK;
}

}  // extern "C"
