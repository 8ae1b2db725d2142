/* libad_b200 -- C ABI of the B200 CUDA device backend.
 *
 * The reference (Eshaancoding/ad) reaches its GPU through per-backend Python
 * helpers over ctypes bindings of libOpenCL / libcuda+libnvrtc.  This library
 * is the single native boundary that replaces those helpers; the Python device
 * class (ad_b200.device.CudaB200Device) binds it with ctypes.  Each
 * declaration names the reference interface it replaces (path:line within the
 * reference project).
 *
 * Conventions: every function returns 0 on success, non-zero on failure with
 * a message in ad_last_error() (thread-local).  Device addresses are uint64_t.
 * Streams are small integers indexing the context's stream table
 * (0 = compute, 1 = host-to-device copies, 2 = device-to-host copies, 3 = comm).
 */
#ifndef AD_B200_H
#define AD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AD_B200_ABI_VERSION 1

typedef struct ad_ctx ad_ctx;
typedef struct ad_kernel ad_kernel;
typedef struct ad_graph ad_graph;

int ad_version(void);
/* cl_helper.py:23-26 check(), cuda_helper.py:14-15 check(): error reporting */
const char* ad_last_error(void);

/* cl_helper.py get_platforms/get_devices/initialize_context/create_command_queue
 * (opencl/device.py:10-44); cuda/device.py:8-19 (cuInit/cuCtxCreate, device 0) */
int ad_device_count(int* n);
int ad_init(int device, int n_streams, ad_ctx** out);
/* opencl/device.py:132-146 __del__ (free_queue/free_context/free_device) */
int ad_destroy(ad_ctx* ctx);
int ad_device_info(ad_ctx* ctx, int* sm_count, int* smem_optin, size_t* free_bytes,
                   size_t* total_bytes);

/* cl_helper.py:151-170 init_buffer; cuda_helper.py:80-84 (cuMemAlloc).  The
 * Python device makes ONE allocation (the arena) and sub-allocates it. */
int ad_malloc(ad_ctx* ctx, size_t bytes, uint64_t* dptr);
/* cl_helper.py free_buffer (opencl/device.py:134-136) */
int ad_free(ad_ctx* ctx, uint64_t dptr);
int ad_memset(ad_ctx* ctx, uint64_t dptr, int value, size_t bytes, int stream);

/* Pinned staging for Feeder/Receiver (the reference copies from pageable numpy
 * memory: cl_helper.py:304-332, cuda_helper.py:86-126) */
int ad_pinned_alloc(size_t bytes, void** p);
int ad_pinned_free(void* p);
/* cl_helper.py:304-332 write_buffer; cuda_helper.py:113-126 (cuMemcpyHtoD at kres offset) */
int ad_h2d(ad_ctx* ctx, uint64_t dst, const void* src, size_t bytes, int stream);
/* cl_helper.py:262-302 read_buffers; cuda_helper.py:86-111 (cuMemcpyDtoH) */
int ad_d2h(ad_ctx* ctx, void* dst, uint64_t src, size_t bytes, int stream);
int ad_d2d(ad_ctx* ctx, uint64_t dst, uint64_t src, size_t bytes, int stream);
/* cl_helper.py:304-332 write_buffer / cuda_helper.py:113-126 with the numpy
 * array's own (pageable) memory as source: staged through a ring of pinned
 * buffers, host copies on a few threads overlapped with the DMA.  Returns once
 * `src` may be reused; the device copy completes in stream order. */
int ad_h2d_pageable(ad_ctx* ctx, uint64_t dst, const void* src, size_t bytes, int stream);
/* cl_helper.py:262-302 read_buffers / cuda_helper.py:86-111 into a pageable
 * (freshly allocated numpy) destination; returns when `dst` holds the data. */
int ad_d2h_pageable(ad_ctx* ctx, void* dst, uint64_t src, size_t bytes, int stream);
/* Host memcpy on the library's copy threads (numpy -> pinned Feeder staging;
 * the reference copies with numpy, cl_helper.py:318-322). */
int ad_host_copy(void* dst, const void* src, size_t bytes);
/* cl_helper.py:457 waitAll (clFinish) */
int ad_stream_sync(ad_ctx* ctx, int stream);
int ad_sync(ad_ctx* ctx);

/* Events: stream ordering between the copy and compute streams, and timing.
 * (The reference has none; its queue-profiling flag is commented out at
 * cl_helper.py:133.) */
int ad_event_create(ad_ctx* ctx, int timing, void** ev);
int ad_event_destroy(void* ev);
int ad_event_record(ad_ctx* ctx, void* ev, int stream);
int ad_stream_wait_event(ad_ctx* ctx, int stream, void* ev);
int ad_event_sync(void* ev);
int ad_event_elapsed_ms(void* start, void* end, float* ms);

/* cl_helper.py:357-384 build_kernel (clCreateProgramWithSource/clBuildProgram);
 * cuda_helper.py:144-198 (nvrtcCompileProgram -> PTX -> cuModuleLoadData).
 * Here NVRTC compiles straight to an sm_100a cubin (no PTX is produced).
 * The returned cubin is malloc'ed; release it with ad_free_host. */
int ad_compile_cubin(const char* src, const char* name, const char* const* opts, int n_opts,
                     void** cubin, size_t* cubin_size, char* log, size_t log_len);
void ad_free_host(void* p);
/* cuda_helper.py:188-198 (cuModuleLoadData + cuModuleGetFunction) */
int ad_load_kernel(ad_ctx* ctx, const void* cubin, const char* fn_name, ad_kernel** out);
/* cl_helper.py free_kernel (opencl/device.py:138-141) */
int ad_kernel_free(ad_kernel* k);
int ad_kernel_set_smem(ad_kernel* k, int bytes);
int ad_kernel_attr(ad_kernel* k, int* regs, int* static_smem, int* max_threads);
/* cl_helper.py:445-455 clEnqueueNDRangeKernel; cuda_helper.py:210-222 cuLaunchKernel.
 * `args` is the usual array of pointers to each kernel parameter. */
int ad_launch(ad_ctx* ctx, ad_kernel* k, unsigned gx, unsigned gy, unsigned gz, unsigned bx,
              unsigned by, unsigned bz, unsigned smem, void** args, int stream);
int ad_check(ad_ctx* ctx);

/* TMA descriptor (CUtensorMap, 128 bytes) for a 2-D row-major tensor; used by
 * the dot-product kernels.  No reference counterpart (the reference's dot
 * product is a scalar loop: opencl/kernels/dotprod.py:7-43). */
int ad_tmap_2d(uint64_t base, uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
               uint32_t box_rows, uint32_t box_cols, int elem_bytes, int swizzle_bytes,
               void* out128);

/* CUDA-graph capture/replay of a ForNode body.  Replaces the Python replay
 * loop of opencl/device.py:114-124 (`for _ in cmd.r: self._run_proc(...)`). */
int ad_graph_begin(ad_ctx* ctx, int stream);
int ad_graph_end(ad_ctx* ctx, int stream, ad_graph** out);
int ad_graph_launch(ad_ctx* ctx, ad_graph* g, int stream);
int ad_graph_destroy(ad_graph* g);

/* NCCL data-parallel gradient all-reduce.  No reference counterpart: the
 * reference has no multi-device code (TODO.md:68-69 lists it as future work).
 * Init is non-blocking and polled against timeout_s; on timeout or error the
 * communicator is aborted and an error returned. */
int ad_nccl_unique_id(void* out128);
int ad_nccl_init(ad_ctx* ctx, int rank, int world, const void* uid128, double timeout_s);
int ad_allreduce_f32(ad_ctx* ctx, uint64_t send, uint64_t recv, size_t count, int op_max,
                     int stream);
int ad_nccl_abort(ad_ctx* ctx);

/* Gradient all-reduce over peer memory (no reference counterpart: the
 * reference has no multi-device code).  ad_peer_init maps every rank's
 * registered region (one cudaMalloc allocation starting at `base`: the
 * device's arena) into every other rank over CUDA IPC, exchanging the handles
 * with one NCCL all-gather (call it on all ranks after ad_nccl_init).
 * ad_peer_allreduce_f32 sums `count` floats at `ptr` (inside the region,
 * 16-byte aligned, count % 4 == 0) over all ranks in place with one kernel:
 * reduce-scatter + all-gather through NVLink loads and stores, ranks meeting
 * at flag barriers.  `op` (0..63) names the call site: each site's calls must
 * come in the same order on every rank.  A barrier that waits more than 2 s
 * writes 7 to the int at `err` (device address) and the kernel returns.
 * ad_peer_close unmaps (also done by ad_destroy). */
int ad_peer_init(ad_ctx* ctx, uint64_t base, size_t bytes);
int ad_peer_allreduce_f32(ad_ctx* ctx, uint64_t ptr, size_t count, int op, int stream, uint64_t err);
int ad_peer_close(ad_ctx* ctx);

/* cudaProfilerStart (on != 0) / cudaProfilerStop: brackets the launches a
 * profiler started with "--profile-from-start off" captures.  No reference
 * counterpart (measurement only). */
int ad_profiler_range(int on);

/* C = A @ B (b_is_nk = 0: B is K x N row-major) or C = A @ B^T (b_is_nk = 1:
 * B is N x K row-major); A is M x K row-major, C is M x N row-major, all fp32
 * device pointers; 3xTF32 on tcgen05.  No counterpart in the reference: this
 * entry point exists for callers that cannot allocate device memory.  It
 * allocates nothing: its split-operand scratch is a fixed 32 MiB device array
 * inside this library, so problems needing more than 8*(Mp+Np)*Kp + 256 bytes
 * of it (Mp = M rounded up to 128, Np = N to 256, Kp = K to 32) are rejected.
 * All calls share that array: calls that overlap on one GPU race.  The first
 * call on each device resolves the array's address (cudaGetSymbolAddress), so
 * make it before any stream capture.  `stream` is a cudaStream_t (NULL = the
 * legacy default stream); the call returns after its work has finished.
 * The resolved address is kept for the life of the process: do not call this
 * on a device after cudaDeviceReset. */
int ad_dot_tf32x3_noalloc(const float* A, const float* B, float* C, int M, int N, int K,
                          int b_is_nk, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AD_B200_H */
