// ad_dot_tf32x3_noalloc: a dense fp32 dot product that allocates nothing.
//
// Some callers cannot allocate device memory at all: code that runs inside a
// host framework which owns every allocation (a memory pool it does not
// share, a fixed pre-planned arena), and code that must not call cudaMalloc
// or cudaFree in its hot loop because those calls synchronise the device.
// This entry point serves them.  It computes C = A @ B (or A @ B^T) with the
// same 3xTF32 tcgen05 scheme as the library's generated dot-product kernels,
// but the split operands (hi/lo TF32 halves, K-major, zero-padded) live in
// the file-scope array below instead of in memory obtained from the caller or
// from cudaMalloc.
//
// Limits and sharing:
//   * The array holds AD_NOALLOC_SCRATCH_BYTES (32 MiB) on every GPU that
//     loads this library, for the life of the process.
//   * A call needs 8 * (Mp + Np) * Kp bytes, Mp = ceil(M/128)*128,
//     Np = ceil(N/256)*256, Kp = ceil(K/32)*32; larger problems are rejected
//     with an error before anything is launched.
//   * Every call uses the same array and leaves its contents behind.  Each
//     call rewrites every element it reads (padding included), and clears its
//     error word before launching, so no state leaks between calls -- but two
//     calls that run at the same time on one GPU (different streams, or
//     different host threads) race on the array.  Serialise them.
//   * The first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (the host-side name of a __device__ array is only a
//     stand-in, not a device address) and raises the kernel's shared-memory
//     limit; make that first call outside any stream capture.
//   * Every call ends by synchronising its stream (it copies the kernel's
//     status word to the host) so that it can report a device-side timeout;
//     it never calls cudaMalloc, cudaFree or any allocating library routine.
//   * The array's address and the shared-memory limit are cached per device
//     for the life of the process; after cudaDeviceReset on a device they are
//     stale, so do not call this entry point on a device that was reset.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/ad_b200.h"

#define AD_NOALLOC_SCRATCH_BYTES (32ull << 20)
#define AD_NA_MAX_DEVICES 64

// The scratch: split operands, then (last 256 bytes) the error word.
static __device__ __align__(256) unsigned char g_noalloc_scratch[AD_NOALLOC_SCRATCH_BYTES];

namespace ad_b200_internal {
void set_error(const char* msg);  // runtime.cu: the message ad_last_error() returns
}

namespace {

struct DevState {
  bool ready = false;
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch on this device
};
DevState g_state[AD_NA_MAX_DEVICES];
std::mutex g_na_mu;

constexpr int NA_BN = 256, NA_STAGES = 2;
constexpr unsigned NA_A_BYTES = 128 * 128, NA_B_BYTES = NA_BN * 128;
constexpr unsigned NA_STAGE_BYTES = 2 * NA_A_BYTES + 2 * NA_B_BYTES;
constexpr int NA_SMEM = NA_STAGES * NA_STAGE_BYTES + 1024 + 256;

__device__ __forceinline__ unsigned na_smem_u32(const void* p) {
  return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ bool na_try(unsigned long long* b, unsigned phase) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(na_smem_u32(b)), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long na_time() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait (2 s): false when the phase never completed.
__device__ __noinline__ bool na_wait(unsigned long long* b, unsigned phase) {
  if (na_try(b, phase)) return true;
  const unsigned long long t0 = na_time();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (na_try(b, phase)) return true;
    if (na_time() - t0 > 2000000000ull) return false;
  }
}
__device__ __forceinline__ unsigned long long na_desc(const void* p) {
  const unsigned long long a = (na_smem_u32(p) >> 4) & 0x3FFFull;
  return a | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// operand(row, k) -> K-major hi/lo halves, zero-padded; `k_contig` says whether
// consecutive k are adjacent in memory (else consecutive rows are).
__global__ void __launch_bounds__(256) na_split(const float* __restrict__ src, long long ld,
                                                int rows, int kdim, int k_contig, int kp,
                                                float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float t[32][33];
  const long long r0 = (long long)blockIdx.y * 32, k0 = (long long)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    if (k_contig) {
      const long long gr = r0 + i, gk = k0 + threadIdx.x;
      t[i][threadIdx.x] = (gr < rows && gk < kdim) ? src[gr * ld + gk] : 0.0f;
    } else {
      const long long gr = r0 + threadIdx.x, gk = k0 + i;
      t[threadIdx.x][i] = (gr < rows && gk < kdim) ? src[gk * ld + gr] : 0.0f;
    }
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const float x = t[i][threadIdx.x];
    unsigned h, l;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
    const float r = x - __uint_as_float(h);
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(r));
    const long long o = (r0 + i) * kp + k0 + threadIdx.x;
    hi[o] = __uint_as_float(h);
    lo[o] = __uint_as_float(l);
  }
}

__global__ void __launch_bounds__(128, 1)
    na_gemm(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
            const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
            float* __restrict__ C, int M, int N, int kblocks, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char na_smem_raw[];
  unsigned char* smem = (unsigned char*)(((unsigned long long)na_smem_raw + 1023) & ~1023ull);
  unsigned long long* full = (unsigned long long*)(smem + NA_STAGES * NA_STAGE_BYTES);
  unsigned long long* empty = full + NA_STAGES;
  unsigned long long* accb = empty + NA_STAGES;
  unsigned* tmem_slot = (unsigned*)(accb + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  volatile int* consumed = abort_flag + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * 128, n0 = blockIdx.x * NA_BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NA_STAGES; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(na_smem_u32(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(na_smem_u32(&empty[s])));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(na_smem_u32(accb)));
    *abort_flag = 0;
    *consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     na_smem_u32(tmem_slot)),
                 "r"(NA_BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const unsigned tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    int issued = 0;
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % NA_STAGES;
      if (kb >= NA_STAGES && !na_wait(&empty[s], ((kb / NA_STAGES) - 1) & 1)) {
        *abort_flag = 1;
        atomicExch(err, 1);
        break;
      }
      if (*abort_flag) break;
      unsigned char* st = smem + s * NA_STAGE_BYTES;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(na_smem_u32(&full[s])),
                   "r"(NA_STAGE_BYTES)
                   : "memory");
      const CUtensorMap* maps[4] = {&tAh, &tAl, &tBh, &tBl};
      const unsigned offs[4] = {0, NA_A_BYTES, 2 * NA_A_BYTES, 2 * NA_A_BYTES + NA_B_BYTES};
      const int rows[4] = {m0, m0, n0, n0};
      for (int q = 0; q < 4; ++q)
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
            "%4}], [%2];" ::"r"(na_smem_u32(st + offs[q])),
            "l"((unsigned long long)maps[q]), "r"(na_smem_u32(&full[s])), "r"(kb * 32), "r"(rows[q])
            : "memory");
      issued = kb + 1;
    }
    if (*abort_flag)
      for (int kb = *consumed; kb < issued; ++kb) na_wait(&full[kb % NA_STAGES], (kb / NA_STAGES) & 1);
  } else if (warp == 1 && lane == 0) {
    constexpr unsigned IDESC =
        (1u << 4) | (2u << 7) | (2u << 10) | ((unsigned)(NA_BN >> 3) << 17) | ((128u >> 4) << 24);
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % NA_STAGES;
      if (!na_wait(&full[s], (kb / NA_STAGES) & 1)) {
        *abort_flag = 1;
        atomicExch(err, 2);
        break;
      }
      if (*abort_flag) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      unsigned char* st = smem + s * NA_STAGE_BYTES;
      const unsigned long long ah = na_desc(st), al = na_desc(st + NA_A_BYTES);
      const unsigned long long bh = na_desc(st + 2 * NA_A_BYTES), bl = na_desc(st + 2 * NA_A_BYTES + NA_B_BYTES);
#pragma unroll
      for (int k8 = 0; k8 < 4; ++k8) {
        const unsigned long long adv = (unsigned long long)(k8 * 32) >> 4;
        const unsigned first = (kb > 0 || k8 > 0) ? 1u : 0u;
        const unsigned long long ad[3] = {ah + adv, ah + adv, al + adv};
        const unsigned long long bd[3] = {bh + adv, bl + adv, bh + adv};
        for (int q = 0; q < 3; ++q)
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
              "l"(ad[q]), "l"(bd[q]), "r"(IDESC), "r"(q == 0 ? first : 1u)
              : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       na_smem_u32(&empty[s]))
                   : "memory");
      *consumed = kb + 1;
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     na_smem_u32(accb))
                 : "memory");
  }
  __syncwarp();

  const bool ok = na_wait(accb, 0);
  if (!ok) atomicExch(err, 3);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();
  if (ok && !*abort_flag) {
    float* tr = (float*)smem + warp * (32 * 33);
    for (int c = 0; c < NA_BN / 32; ++c) {
      unsigned r[32];
      const unsigned taddr = tmem + ((unsigned)(warp * 32) << 16) + (unsigned)(c * 32);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
          "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
            "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
            "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
            "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
            "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int j = 0; j < 32; ++j) tr[lane * 33 + j] = __uint_as_float(r[j]);
      __syncwarp();
      for (int i = 0; i < 32; ++i) {
        const long long om = (long long)m0 + warp * 32 + i;
        const long long on = (long long)n0 + c * 32 + lane;
        if (om < M && on < N) C[om * N + on] = tr[i * 33 + lane];
      }
      __syncwarp();
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NA_BN) : "memory");
}

int na_fail(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  ad_b200_internal::set_error(buf);
  return 1;
}

long long pad(long long x, long long m) { return (x + m - 1) / m * m; }

}  // namespace

extern "C" int ad_dot_tf32x3_noalloc(const float* A, const float* B, float* C, int M, int N, int K,
                                     int b_is_nk, void* stream) {
  if (!A || !B || !C) return na_fail("ad_dot_tf32x3_noalloc: null operand");
  if (M <= 0 || N <= 0 || K <= 0) return na_fail("ad_dot_tf32x3_noalloc: empty shape %d x %d x %d", M, N, K);
  const long long Mp = pad(M, 128), Np = pad(N, NA_BN), Kp = pad(K, 32);
  const unsigned long long need = 8ull * (unsigned long long)(Mp + Np) * (unsigned long long)Kp;
  if (need + 256 > AD_NOALLOC_SCRATCH_BYTES)
    return na_fail(
        "ad_dot_tf32x3_noalloc: %d x %d x %d needs %llu bytes of scratch; the fixed array holds %llu "
        "(8 * (Mp + Np) * Kp + 256 must fit)",
        M, N, K, need + 256, (unsigned long long)AD_NOALLOC_SCRATCH_BYTES);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return na_fail("cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= AD_NA_MAX_DEVICES) return na_fail("ad_dot_tf32x3_noalloc: device index %d out of range", dev);
  {
    // once per device, with that device current: resolve the array's device address
    std::lock_guard<std::mutex> lk(g_na_mu);
    DevState& st = g_state[dev];
    if (!st.ready) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return na_fail("cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      e = cudaFuncSetAttribute(na_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, NA_SMEM);
      if (e != cudaSuccess) return na_fail("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      st.scratch = static_cast<unsigned char*>(p);
      st.ready = true;
    }
  }
  unsigned char* base = g_state[dev].scratch;
  float* a_hi = reinterpret_cast<float*>(base);
  float* a_lo = a_hi + Mp * Kp;
  float* b_hi = a_lo + Mp * Kp;
  float* b_lo = b_hi + Np * Kp;
  int* err = reinterpret_cast<int*>(base + AD_NOALLOC_SCRATCH_BYTES - 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  alignas(64) unsigned char maps[4][128];
  const uint64_t addrs[4] = {(uint64_t)a_hi, (uint64_t)a_lo, (uint64_t)b_hi, (uint64_t)b_lo};
  const uint64_t rows[4] = {(uint64_t)Mp, (uint64_t)Mp, (uint64_t)Np, (uint64_t)Np};
  const uint32_t box[4] = {128, 128, NA_BN, NA_BN};
  for (int q = 0; q < 4; ++q)
    if (ad_tmap_2d(addrs[q], rows[q], (uint64_t)Kp, 4ull * Kp, box[q], 32, 4, 128, maps[q]) != 0)
      return na_fail("ad_dot_tf32x3_noalloc: tensor map: %s", ad_last_error());

  e = cudaMemsetAsync(err, 0, sizeof(int), s);
  if (e != cudaSuccess) return na_fail("cudaMemsetAsync: %s", cudaGetErrorString(e));
  dim3 sb(32, 8);
  na_split<<<dim3((unsigned)(Kp / 32), (unsigned)(Mp / 32)), sb, 0, s>>>(A, K, M, K, 1, (int)Kp, a_hi, a_lo);
  if (b_is_nk)
    na_split<<<dim3((unsigned)(Kp / 32), (unsigned)(Np / 32)), sb, 0, s>>>(B, K, N, K, 1, (int)Kp, b_hi, b_lo);
  else
    na_split<<<dim3((unsigned)(Kp / 32), (unsigned)(Np / 32)), sb, 0, s>>>(B, N, N, K, 0, (int)Kp, b_hi, b_lo);
  na_gemm<<<dim3((unsigned)(Np / NA_BN), (unsigned)(Mp / 128)), 128, NA_SMEM, s>>>(
      *reinterpret_cast<CUtensorMap*>(maps[0]), *reinterpret_cast<CUtensorMap*>(maps[1]),
      *reinterpret_cast<CUtensorMap*>(maps[2]), *reinterpret_cast<CUtensorMap*>(maps[3]), C, M, N,
      (int)(Kp / 32), err);
  e = cudaGetLastError();
  if (e != cudaSuccess) return na_fail("launch: %s", cudaGetErrorString(e));
  int h_err = 0;
  e = cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return na_fail("ad_dot_tf32x3_noalloc: %s", cudaGetErrorString(e));
  if (h_err) return na_fail("ad_dot_tf32x3_noalloc: device-side wait expired (code %d)", h_err);
  return 0;
}
