/* tallymap_b200: the C ABI of the B200 kernel backend for tallymap.
 *
 * This is the drop-in boundary below tallymap's kernel-backend driver.  In the reference the driver
 * (tallymap/backends/kernel/__init__.py:135-185, KB.run) reaches the device through ONE XLA FFI custom call,
 * "tallymap_cuda_launch", handled by tallymap/backends/kernel/shim.cc; the entry points below are what that shim
 * exports and what its handler does, as plain C: pointers, sizes and a stream, no XLA, JAX or torch types.
 *
 * Buffers: every launch takes ONE array of device pointers, the program's inputs first (per-item operands,
 * broadcast operands, hoisted constants, the optional item claim order), then its results (sum tallies, scratch accumulators, the control words,
 * stats int32[5], per-item results) -- the order of the reference's SjParams (backends/kernel/kernel.py:570-596).
 * The first n_zero results are zeroed on the stream before the kernel runs (shim.cc:210-219).
 *
 * Errors: every entry point returns 0 on success and a nonzero TM_E* code otherwise; tm_last_error() returns the
 * calling thread's last message.  Launches are asynchronous on the caller's stream; nothing here synchronises.
 */
#ifndef TALLYMAP_B200_H
#define TALLYMAP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TM_OK = 0,
  TM_EINVAL = 1,   /* bad id, buffer count, size or pointer (the FFI handler's kInvalidArgument) */
  TM_ECUDA = 2,    /* a CUDA runtime call failed (kInternal); the message names it */
  TM_EDEVICE = 3   /* tm_check_status: the device error word of a finished launch is set */
};

/* ABI version of this header (bumped on any signature or buffer-layout change). */
int tm_abi_version(void);

/* The calling thread's last error message ("" when none). */
const char* tm_last_error(void);

/* Look up a built-in (ahead-of-time compiled, sm_100a) kernel by program name, e.g. "rw_fwd", "rw_grad".
 * *id receives its kernel id; *n_buffers the number of buffer pointers a launch takes (may be NULL).
 * Replaces: the kernel cache lookup of backends/kernel/__init__.py:106-128 (kernel(), keyed by a digest). */
int tm_kernel_id(const char* name, int64_t* id, int32_t* n_buffers);

/* Enumerate the built-in kernels: *name receives the i-th name (NULL past the end). */
int tm_kernel_name(int32_t i, const char** name);

/* Register a kernel image (a cubin or fatbin for sm_100a containing `extern "C" __global__ tm_main(Params, int64)`,
 * from the runtime lowering) under `id`; re-registering an id keeps the first image.  The image is copied and loaded
 * lazily on each device at its first launch.  n_buffers: the pointers a launch takes; smem_bytes: its dynamic shared
 * memory; block: threads per block.
 * Replaces: tallymap_register (backends/kernel/shim.cc:134-142). */
int tm_register(int64_t id, const void* image, size_t n, const char* note, int32_t n_buffers, int32_t smem_bytes,
                int32_t block);

/* Compile a lowered item program for sm_100a with NVRTC (libnvrtc.so.12, loaded on first use) and register it as
 * tm_register does: `source` is CUDA C++ that includes the runtime headers found in `include_dir` and defines
 * `extern "C" __global__ void tm_main(tmb::Params, long long)`.  Compiled with -arch=sm_100a -std=c++17 --fmad=false
 * -lineinfo.  On a compile error returns TM_EINVAL with the NVRTC log in tm_last_error().
 * Replaces: compile_cubin + tallymap_register (backends/kernel/compile.py:160-173, shim.cc:134-142). */
int tm_compile_register(int64_t id, const char* source, const char* include_dir, const char* note,
                        int32_t n_buffers, int32_t smem_bytes, int32_t block);

/* Compile as tm_compile_register does, without registering: the cubin's size into *n and, when `out` holds cap >= *n
 * bytes, the cubin itself (call once with out = NULL for the size).  For a caller that keeps compiled items on disk
 * and registers them later with tm_register (the reference's disk cubin cache, backends/kernel/__init__.py:71-128).
 *   flags: bit 0 (TM_COMPILE_FMAD): FMA contraction of float multiply-adds (--fmad=true), the reference's
 *          cuda_math='fast' (backends/kernel/__init__.py:141-146); 0: --fmad=false, as tm_compile_register */
#define TM_COMPILE_FMAD 1
int tm_compile(const char* source, const char* include_dir, int32_t block, int32_t flags, void* out, size_t cap,
               size_t* n);

/* Bytes of one stored loop state in a built-in replay program's scratch (the size the host multiplies by the states
 * per thread and the threads to allocate it; 0 for a program with no replay scratch).  No device access.
 * (No counterpart in the reference: its scratch sizes come from the generated source's layout.) */
int tm_kernel_state_bytes(int64_t id, int32_t* bytes);

/* Resources of a kernel on the current device: out[7] = registers per thread, local bytes per thread, static
 * shared bytes per block, resident blocks per SM, SMs, max resident threads per SM, block size.
 * Replaces: tallymap_kernel_info (backends/kernel/shim.cc:147-155). */
int tm_kernel_info(int64_t id, long long* out);

/* 1 when this build carries the XLA FFI handler `TallymapB200Launch` (tallymap_b200/csrc/tm_ffi.cc, compiled where
 * XLA's FFI headers were on the include path), 0 otherwise.  The handler is the custom-call target a JAX install
 * registers (jax.ffi.register_ffi_target(..., jax.ffi.pycapsule(lib.TallymapB200Launch), platform="CUDA")) with the
 * reference's attributes kernel_id (int64), block (int32, checked against the kernel's registered block), n_zero
 * (int32), flags (int32) and n_items (int64), and calls tm_launch on XLA's stream.
 * Replaces: the XLA FFI handler symbol TallymapLaunch (backends/kernel/shim.cc:241-250). */
int tm_ffi_available(void);

/* Launch kernel `id` on `stream` (a cudaStream_t; NULL = the legacy default stream) over n_items items.
 *   bufs[n_args + n_rets]: device pointers, inputs then results; ret_bytes[n_rets]: each result's size in bytes
 *   n_zero: the first n_zero results are zeroed (cudaMemsetAsync on `stream`) before the launch
 *   flags: bit 2 (4): the grid is not capped by n_items (a program that spawns children); bit 3 (8): the last
 *          argument is the program's optional item claim order (int32[n_items] permutation) and may be NULL
 *   status: optional (may be NULL); receives the cudaError_t of the launch (0: launched)
 * The grid is one persistent block per resident slot (SMs x blocks per SM at the kernel's occupancy), capped at
 * ceil(n_items / block).
 * Replaces: the body of the XLA FFI handler SjLaunchImpl (backends/kernel/shim.cc:157-239). */
int tm_launch(int64_t id, void* stream, void* const* bufs, int32_t n_args, int32_t n_rets, const size_t* ret_bytes,
              int32_t n_zero, int32_t flags, int64_t n_items, int32_t* status);

/* The cross-GPU step of an exact f32 tally (TSpec.exact): `words` holds n_src exact scratch buffers end to end
 * (each: n_bins x 5 int64 carry-save words, then one uint32 flag per bin packed into (n_bins + 1) / 2 uint64), e.g.
 * every rank's buffer after an all-gather; out[n_bins] receives the correctly rounded f32 of the exact total (NaN
 * for a flagged or overflowing bin, counted in stats[3]).
 * Replaces: the psum of a kernel-backend call's tallies under sharding (tallymap/_primitive.py:245-262), for the
 * exact cotangent tallies whose words cannot be summed word by word without carries. */
int tm_exact_combine(void* stream, const void* words, int32_t n_src, int32_t n_bins, float* out, int32_t* stats);

/* Exact f32 scatter-add: out[b] = the correctly rounded sum of every vals[i] with bins[i] == b (out-of-range bins
 * dropped and counted in stats[4]; non-finite values make their bin NaN, counted in stats[3]).  `words` is caller
 * scratch of (n_bins x 5 + (n_bins + 1) / 2) uint64, zeroed here.
 * Replaces: the exact accumulator of a Sum(fixed_point=True) float32 output (backends/kernel/kernel.py:870-941,
 * DENSE), on its own. */
int tm_exact_scatter(void* stream, const float* vals, const int32_t* bins, int64_t n, int32_t n_bins, void* words,
                     float* out, int32_t* stats);

/* tm_exact_scatter without scratch from the caller and without any device allocation.  Some callers cannot
 * allocate: an XLA FFI handler, whose device memory belongs to XLA's pool (JAX preallocates most of the GPU, and a
 * cudaMalloc beside it can fail or fragment memory), and any caller on a path that must not block, since cudaMalloc
 * and cudaFree may synchronise the device.  This variant keeps its scratch words in a fixed device array inside the
 * library instead, at most 65,536 bins (2.75 MiB, held by every GPU that loads the library until the process exits);
 * a larger n_bins is rejected with TM_EINVAL.  The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before any stream capture.  Each call clears
 * the words it uses, so consecutive calls are independent, but every call on a device shares that device's copy of
 * the array: calls on one device that can overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller (calls on different devices do not race).  The looked-up address lives as long as the
 * device's primary context: after cudaDeviceReset of that device, do not call this entry point again in the process.
 * (No counterpart in the reference: its handler receives every scratch buffer from XLA.) */
int tm_exact_scatter_noalloc(void* stream, const float* vals, const int32_t* bins, int64_t n, int32_t n_bins,
                             float* out, int32_t* stats);

/* Generation lists of a recorded spawn tree, the launch order of the tree adjoint (replaces the XLA ordering of
 * tallymap/_reverse_spawn.py:255-283 inside tree_vjp; the adjoint launches themselves go through tm_launch with the
 * generation's list as the claim order).  `records`: n_records records of record_bytes bytes, each with its
 * generation at byte gen_offset, an integer of gen_bytes bytes (2: uint16, 4: int32) -- a record array, or a compact
 * array of generations (record_bytes = gen_bytes, gen_offset = 0).  On `stream`: counts[g] (uint64[n_gen + 1]) = the
 * records of generation g, with generations outside [0, n_gen) counted in counts[n_gen] and listed nowhere; lists
 * (int32[n_records]) = the record indices grouped by generation, generation g at [sum(counts[:g]),
 * sum(counts[:g + 1])), in no particular order within a generation; cursor (uint64[n_gen + 1]) is scratch.
 * n_gen <= TM_TREE_MAX_GEN, n_records < 2^31. */
#define TM_TREE_MAX_GEN 8192
int tm_tree_generations(void* stream, const void* records, int64_t n_records, int32_t record_bytes,
                        int32_t gen_offset, int32_t gen_bytes, int32_t n_gen, uint64_t* counts, uint64_t* cursor,
                        int32_t* lists);

/* Calibration probe for rooflines: `iters` threefry2x32 evaluations per thread on every resident thread slot of
 * the device (at most out_len threads, a multiple of 128), no memory traffic besides one word per thread.
 * *threads_used receives the thread count.  Time it on `stream` for the device's threefry issue rate.
 * (No counterpart in the reference, which reports no rooflines.) */
int tm_probe_threefry(void* stream, int32_t iters, uint32_t* out, int64_t out_len, int64_t* threads_used);

/* Issue-rate probes for rooflines, launched like tm_probe_threefry on every resident thread slot (at most out_len
 * threads), `iters` iterations per thread, register-resident, no memory traffic besides one word per thread:
 *   kind 0  one threefry2x32 per iteration (the walkers' dominant operation; = tm_probe_threefry)
 *   kind 1  16 FP32 instructions per iteration (8 independent multiply and add chains): the FP32 issue rate
 *   kind 2  one trial step of the Lorenz RK45 item per iteration (its own instruction mix at its own occupancy)
 *   kind 3  one trial step and one step VJP of that item per iteration (the replay's sweep mix)
 *   kind 4  one step of the photon-slab item per iteration (its draws, path, voxel, scattering and roulette; the
 *           deposit summed in a register)
 *   kind 5  one trial step of the Lorenz RK45 item with its stages' tangents per iteration (the one-pass forward-mode
 *           program's step)
 * (No counterpart in the reference, which reports no rooflines.) */
int tm_probe_issue(void* stream, int32_t kind, int32_t iters, uint32_t* out, int64_t out_len,
                   int64_t* threads_used);

/* The backend's f32 math on the device, elementwise: fn 0 log, 1 exp, 2 sin, 3 cos, 4 pow(x, y), 5 atan,
 * 6 atan2(x, y) (x the ordinate), 7 asin, 8 acos, 9 tan, 10 sinh, 11 cosh, 12 asinh, 13 acosh, 14 atanh, 15 exp2,
 * 16 log2, 17 cbrt, 18 erf, 19 erfc, 20 erfinv (y read only by pow and atan2).
 * The item programs use this math on the device and the same code on the host, so the two agree bitwise; this entry
 * point lets a caller check that.  (The reference has no counterpart: its device math is libdevice, its host math
 * libm, backends/kernel/kernel.py:29-57, host.py:9-11.) */
int tm_math_eval(void* stream, int32_t fn, const float* x, const float* y, float* out, int64_t n);

/* Read a finished launch's device error word (ctl[3] of its control-word buffer, host-visible copy `ctl_host`,
 * 8 uint32 words).  Returns TM_OK when it is clear, TM_EDEVICE (with a message) when a device-side wait gave up or
 * a bounds check failed. */
int tm_check_status(const uint32_t* ctl_host);

#ifdef __cplusplus
}
#endif

#endif /* TALLYMAP_B200_H */
