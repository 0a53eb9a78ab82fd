// The C ABI of the tallymap B200 backend (include/tallymap_b200.h): kernel registry, launcher, resource query.
//
// The reference reaches the device through one XLA FFI handler (tallymap/backends/kernel/shim.cc:157-239) that
// loads NVRTC modules per context, zeroes the first n_zero results, sizes a persistent grid by occupancy and
// launches on XLA's stream.  Here the same contract is plain C over the CUDA runtime: built-in kernels are compiled
// ahead of time for sm_100a into this library; runtime-lowered images are registered as cubins and loaded through
// the context-independent library API (cudaLibraryLoadData), so no per-context bookkeeping is needed.
#include <cuda_runtime.h>

#include <dlfcn.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/tallymap_b200.h"
#include "items_ode.cuh"
#include "items_photon.cuh"
#include "items_shower.cuh"
#include "items_walks.cuh"
#include "tm_aux.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(const char* what, cudaError_t e) {
  return fail(TM_ECUDA, "tallymap_b200: %s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// FNV-1a of a name: the id of a built-in kernel (stable across builds, distinct from registered image ids only by
// convention: registered ids come from an image digest)
int64_t name_id(const char* s) {
  uint64_t h = 1469598103934665603ull;
  for (; *s; ++s) h = (h ^ (unsigned char)*s) * 1099511628211ull;
  return (int64_t)(h & 0x7fffffffffffffffull);
}

struct Kernel {
  std::string name;
  const void* fn = nullptr;         // built-in: the __global__ function; registered: the cudaKernel_t
  int nbuf = 0, smem = 0, block = TM_BLOCK;
  int state_bytes = 0;              // a replay program: bytes of one stored loop state in its scratch
  std::string image, note;          // registered images only
  cudaLibrary_t lib = nullptr;
  std::unordered_map<int, int> occ; // device -> resident blocks per SM
};

std::mutex g_mu;
std::unordered_map<int64_t, Kernel>* g_reg = nullptr;
std::vector<std::string>* g_names = nullptr;

template <class I>
void add_forward(const char* name) {
  Kernel k;
  k.name = name;
  if constexpr (tmb::min_blocks_of<I>::value > 0) k.fn = reinterpret_cast<const void*>(&tmb::forward_kernel_occ<I>);
  else k.fn = reinterpret_cast<const void*>(&tmb::forward_kernel<I>);
  k.nbuf = I::kNBuf;
  k.smem = I::kSmemBytes;
  k.block = tmb::block_of<I>::value;
  (*g_reg)[name_id(name)] = k;
  g_names->push_back(name);
}

template <class I>
void add_spawn(const char* name) {
  Kernel k;
  k.name = name;
  k.fn = reinterpret_cast<const void*>(&tmb::spawn_kernel<I>);
  k.nbuf = I::kNBuf;
  k.smem = tmb::SpawnSmem<I>::kBytes;         // the item's block, then the lanes' shared stack entries
  (*g_reg)[name_id(name)] = k;
  g_names->push_back(name);
}

template <class I, int V>
void add_vg(const char* name) {
  Kernel k;
  k.name = name;
  k.fn = reinterpret_cast<const void*>(&tmb::vg_kernel<I, V>);
  k.nbuf = I::kNBuf;
  k.smem = I::kSmemBytes;
  k.state_bytes = (int)sizeof(typename I::Stored);
  (*g_reg)[name_id(name)] = k;
  g_names->push_back(name);
}

template <class I, int V>
void add_replay(const char* name) {
  Kernel k;
  k.name = name;
  if constexpr (tmb::min_blocks_of<I>::value > 0) k.fn = reinterpret_cast<const void*>(&tmb::replay_kernel_occ<I, V>);
  else k.fn = reinterpret_cast<const void*>(&tmb::replay_kernel<I, V>);
  k.nbuf = I::kNBuf;
  k.smem = I::kSmemBytes;
  k.state_bytes = (int)sizeof(typename I::Stored);
  (*g_reg)[name_id(name)] = k;
  g_names->push_back(name);
}

// the built-in programs; the replay adjoints apply up to 4 step VJPs per iteration (their checkpoint count C is a
// launch constant)
void init_registry() {
  if (g_reg) return;
  g_reg = new std::unordered_map<int64_t, Kernel>();
  g_names = new std::vector<std::string>();
  add_forward<tmb::Q1Fwd>("q1_fwd");
  add_replay<tmb::Q1Grad, 4>("q1_grad");
  add_forward<tmb::RWFwd>("rw_fwd");
  add_replay<tmb::RWGrad, 4>("rw_grad");
  add_vg<tmb::Q1VG, 4>("q1_vg");
  add_vg<tmb::RWVG, 4>("rw_vg");
  add_replay<tmb::Q1VG, 4>("q1_vg_replay");
  add_replay<tmb::RWVG, 4>("rw_vg_replay");
  add_forward<tmb::Q1VG1>("q1_vg_onepass");
  add_forward<tmb::RWVG1>("rw_vg_onepass");
  add_forward<tmb::PHFwd>("ph_fwd");
  add_replay<tmb::PHGrad, 1>("ph_grad");
  add_forward<tmb::PHVG1>("ph_vg_onepass");
  add_forward<tmb::ODFwd>("od_fwd");
  add_replay<tmb::ODGrad, 1>("od_grad");
  add_forward<tmb::ODVG1>("od_vg_onepass");
  add_spawn<tmb::SHFwd>("sh_fwd");
  add_spawn<tmb::SHRec>("sh_rec");
  add_spawn<tmb::SHVG1>("sh_vg_onepass");
  add_replay<tmb::SHGrad, 1>("sh_grad");
}

Kernel* find(int64_t id) {
  init_registry();
  auto it = g_reg->find(id);
  return it == g_reg->end() ? nullptr : &it->second;
}

// load a registered image on first use (library API: valid in every context of the process)
int ensure_loaded(Kernel& k) {
  if (k.fn) return TM_OK;
  cudaError_t e = cudaLibraryLoadData(&k.lib, k.image.data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
  if (e != cudaSuccess) return cuda_fail("cudaLibraryLoadData", e);
  cudaKernel_t kern = nullptr;
  e = cudaLibraryGetKernel(&kern, k.lib, "tm_main");
  if (e != cudaSuccess) return cuda_fail("cudaLibraryGetKernel(tm_main)", e);
  k.fn = reinterpret_cast<const void*>(kern);
  return TM_OK;
}

int occupancy(Kernel& k, int dev, int* occ) {
  auto it = k.occ.find(dev);
  if (it != k.occ.end()) { *occ = it->second; return TM_OK; }
  // a block's static shared memory (e.g. the end-of-launch compaction pool) and its dynamic shared memory together
  // past the 48 KiB default need the opt-in
  cudaFuncAttributes fa;
  cudaError_t ea = cudaFuncGetAttributes(&fa, k.fn);
  if (ea != cudaSuccess) return cuda_fail("cudaFuncGetAttributes", ea);
  if (k.smem + fa.sharedSizeBytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
    if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute", e);
  }
  int o = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k.fn, k.block, (size_t)k.smem);
  if (e != cudaSuccess) return cuda_fail("cudaOccupancyMaxActiveBlocksPerMultiprocessor", e);
  if (o < 1) o = 1;
  k.occ[dev] = o;
  *occ = o;
  return TM_OK;
}

// ------------------------------------------------------------------------------------------------ no-alloc scratch
// Scratch of tm_exact_scatter_noalloc: the exact words of at most TM_NOALLOC_MAX_BINS bins, in a fixed device array
// that every GPU loading this library holds until the process exits (2.75 MiB).  Host code must not pass the array's
// name to a kernel (on the host it is a stand-in, not a device address): noalloc_words() looks up its device address
// once per device, with that device current, and caches it.  Each device holds its own copy of the array, so the
// cached address belongs to that device's primary context: it stays valid until the process exits, unless the
// process calls cudaDeviceReset on that device, which destroys the context and the array with it (after such a reset
// this entry point must not be called again in the process).
#define TM_NOALLOC_MAX_BINS 65536
static __device__ __align__(256) unsigned long long
    g_noalloc_words[(size_t)TM_NOALLOC_MAX_BINS * tmb::kExactWords + (TM_NOALLOC_MAX_BINS + 1) / 2];

#define TM_NOALLOC_MAX_DEVICES 64
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[TM_NOALLOC_MAX_DEVICES] = {};

int noalloc_words(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= TM_NOALLOC_MAX_DEVICES)
    return fail(TM_EINVAL, "tallymap_b200: device %d is beyond the %d devices the fixed scratch serves", dev,
                TM_NOALLOC_MAX_DEVICES);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_words);
    if (e != cudaSuccess) return cuda_fail("cudaGetSymbolAddress(fixed scratch)", e);
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return TM_OK;
}

}  // namespace

extern "C" {

int tm_abi_version(void) { return 1; }

const char* tm_last_error(void) { return g_err.c_str(); }

int tm_kernel_id(const char* name, int64_t* id, int32_t* n_buffers) {
  if (!name || !id) return fail(TM_EINVAL, "tallymap_b200: tm_kernel_id: null argument");
  std::lock_guard<std::mutex> lk(g_mu);
  Kernel* k = find(name_id(name));
  if (!k || k->name != name) return fail(TM_EINVAL, "tallymap_b200: no built-in kernel named '%s'", name);
  *id = name_id(name);
  if (n_buffers) *n_buffers = k->nbuf;
  return TM_OK;
}

int tm_kernel_name(int32_t i, const char** name) {
  if (!name) return fail(TM_EINVAL, "tallymap_b200: tm_kernel_name: null argument");
  std::lock_guard<std::mutex> lk(g_mu);
  init_registry();
  *name = (i >= 0 && (size_t)i < g_names->size()) ? (*g_names)[i].c_str() : nullptr;
  return TM_OK;
}

int tm_register(int64_t id, const void* image, size_t n, const char* note, int32_t n_buffers, int32_t smem_bytes,
                int32_t block) {
  if (!image || n == 0) return fail(TM_EINVAL, "tallymap_b200: tm_register: empty image");
  if (n_buffers <= 0 || n_buffers > TM_MAXP)
    return fail(TM_EINVAL, "tallymap_b200: tm_register: %d buffers (1..%d allowed)", n_buffers, TM_MAXP);
  if (block <= 0 || block > 1024 || block % 32)
    return fail(TM_EINVAL, "tallymap_b200: tm_register: block %d is not a multiple of 32 in 32..1024", block);
  std::lock_guard<std::mutex> lk(g_mu);
  init_registry();
  Kernel& k = (*g_reg)[id];
  if (!k.image.empty() || k.fn) return TM_OK;   // first registration wins (shim.cc:134-142)
  k.name = note ? note : "";
  k.image.assign(static_cast<const char*>(image), n);
  k.note = k.name;
  k.nbuf = n_buffers;
  k.smem = smem_bytes;
  k.block = block;
  return TM_OK;
}

// ------------------------------------------------------------------------------------------------ NVRTC
// libnvrtc is opened on first use (the library itself does not link it, so it loads where NVRTC is absent)
namespace {
struct Nvrtc {
  void* h = nullptr;
  int (*create)(void**, const char*, const char*, int, const char* const*, const char* const*) = nullptr;
  int (*compile)(void*, int, const char* const*) = nullptr;
  int (*log_size)(void*, size_t*) = nullptr;
  int (*log)(void*, char*) = nullptr;
  int (*cubin_size)(void*, size_t*) = nullptr;
  int (*cubin)(void*, char*) = nullptr;
  int (*destroy)(void**) = nullptr;
};
Nvrtc g_nvrtc;

int load_nvrtc() {
  if (g_nvrtc.h) return TM_OK;
  const char* names[] = {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"};
  void* h = nullptr;
  for (const char* n : names)
    if ((h = dlopen(n, RTLD_NOW | RTLD_LOCAL))) break;
  if (!h) return fail(TM_EINVAL, "tallymap_b200: NVRTC (libnvrtc.so.12) is not available: %s", dlerror());
  Nvrtc f;
  f.h = h;
  f.create = reinterpret_cast<decltype(f.create)>(dlsym(h, "nvrtcCreateProgram"));
  f.compile = reinterpret_cast<decltype(f.compile)>(dlsym(h, "nvrtcCompileProgram"));
  f.log_size = reinterpret_cast<decltype(f.log_size)>(dlsym(h, "nvrtcGetProgramLogSize"));
  f.log = reinterpret_cast<decltype(f.log)>(dlsym(h, "nvrtcGetProgramLog"));
  f.cubin_size = reinterpret_cast<decltype(f.cubin_size)>(dlsym(h, "nvrtcGetCUBINSize"));
  f.cubin = reinterpret_cast<decltype(f.cubin)>(dlsym(h, "nvrtcGetCUBIN"));
  f.destroy = reinterpret_cast<decltype(f.destroy)>(dlsym(h, "nvrtcDestroyProgram"));
  if (!f.create || !f.compile || !f.log_size || !f.log || !f.cubin_size || !f.cubin || !f.destroy)
    return fail(TM_EINVAL, "tallymap_b200: libnvrtc lacks an entry point");
  g_nvrtc = f;
  return TM_OK;
}
}  // namespace

// NVRTC for sm_100a: the cubin of `source` into *cubin (the log in tm_last_error on failure)
static int compile_cubin(const char* source, const char* include_dir, const char* note, int32_t block, int32_t flags,
                         std::vector<char>* cubin) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = load_nvrtc();
    if (rc) return rc;
  }
  void* prog = nullptr;
  if (g_nvrtc.create(&prog, source, "tm_item.cu", 0, nullptr, nullptr) != 0 || !prog)
    return fail(TM_EINVAL, "tallymap_b200: nvrtcCreateProgram failed");
  const std::string inc = std::string("-I") + include_dir;
  char blk[32];
  std::snprintf(blk, sizeof(blk), "-DTM_BLOCK=%d", block);
  const char* fmad = (flags & 1) ? "--fmad=true" : "--fmad=false";
  const char* opts[] = {"-arch=sm_100a", "-std=c++17", fmad, "-lineinfo", inc.c_str(), "-I/usr/local/cuda/include", blk};
  const int crc = g_nvrtc.compile(prog, 7, opts);
  if (crc != 0) {
    size_t n = 0;
    g_nvrtc.log_size(prog, &n);
    std::string log(n, '\0');
    if (n) g_nvrtc.log(prog, &log[0]);
    g_nvrtc.destroy(&prog);
    return fail(TM_EINVAL, "tallymap_b200: NVRTC failed to compile '%s':\n%.3000s", note ? note : "", log.c_str());
  }
  size_t n = 0;
  g_nvrtc.cubin_size(prog, &n);
  cubin->assign(n, 0);
  if (n) g_nvrtc.cubin(prog, cubin->data());
  g_nvrtc.destroy(&prog);
  if (n == 0) return fail(TM_EINVAL, "tallymap_b200: NVRTC produced no cubin");
  return TM_OK;
}

int tm_compile_register(int64_t id, const char* source, const char* include_dir, const char* note,
                        int32_t n_buffers, int32_t smem_bytes, int32_t block) {
  if (!source || !include_dir) return fail(TM_EINVAL, "tallymap_b200: tm_compile_register: null argument");
  {
    std::lock_guard<std::mutex> lk(g_mu);
    init_registry();
    if (find(id)) return TM_OK;       // already registered (first registration wins)
  }
  std::vector<char> cubin;
  const int rc = compile_cubin(source, include_dir, note, block, 0, &cubin);
  if (rc) return rc;
  return tm_register(id, cubin.data(), cubin.size(), note, n_buffers, smem_bytes, block);
}

int tm_compile(const char* source, const char* include_dir, int32_t block, int32_t flags, void* out, size_t cap,
               size_t* n) {
  if (!source || !include_dir || !n) return fail(TM_EINVAL, "tallymap_b200: tm_compile: null argument");
  if (flags & ~1) return fail(TM_EINVAL, "tallymap_b200: tm_compile: unknown flags %d", (int)flags);
  std::vector<char> cubin;
  const int rc = compile_cubin(source, include_dir, "item", block, flags, &cubin);
  if (rc) return rc;
  *n = cubin.size();
  if (out && cap >= cubin.size()) std::memcpy(out, cubin.data(), cubin.size());
  return TM_OK;
}

int tm_kernel_state_bytes(int64_t id, int32_t* bytes) {
  if (!bytes) return fail(TM_EINVAL, "tallymap_b200: tm_kernel_state_bytes: null argument");
  std::lock_guard<std::mutex> lk(g_mu);
  Kernel* k = find(id);
  if (!k) return fail(TM_EINVAL, "tallymap_b200: kernel id %lld is not registered", (long long)id);
  *bytes = k->state_bytes;
  return TM_OK;
}

int tm_kernel_info(int64_t id, long long* out) {
  if (!out) return fail(TM_EINVAL, "tallymap_b200: tm_kernel_info: null argument");
  std::lock_guard<std::mutex> lk(g_mu);
  Kernel* k = find(id);
  if (!k) return fail(TM_EINVAL, "tallymap_b200: kernel id %lld is not registered", (long long)id);
  int rc = ensure_loaded(*k);
  if (rc) return rc;
  int dev = 0, sms = 0, per_sm = 0, occ = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
  if ((rc = occupancy(*k, dev, &occ))) return rc;
  cudaFuncAttributes a;
  e = cudaFuncGetAttributes(&a, k->fn);
  if (e != cudaSuccess) return cuda_fail("cudaFuncGetAttributes", e);
  const long long v[7] = {a.numRegs, (long long)a.localSizeBytes, (long long)a.sharedSizeBytes, occ, sms, per_sm,
                          k->block};
  for (int i = 0; i < 7; ++i) out[i] = v[i];
  return TM_OK;
}

int tm_launch(int64_t id, void* stream, void* const* bufs, int32_t n_args, int32_t n_rets, const size_t* ret_bytes,
              int32_t n_zero, int32_t flags, int64_t n_items, int32_t* status) {
  if (status) *status = 0;
  if (!bufs || (n_rets > 0 && !ret_bytes)) return fail(TM_EINVAL, "tallymap_b200: tm_launch: null buffer list");
  if (n_items < 0) return fail(TM_EINVAL, "tallymap_b200: tm_launch: n_items %lld < 0", (long long)n_items);
  if (n_zero < 0 || n_zero > n_rets) return fail(TM_EINVAL, "tallymap_b200: tm_launch: n_zero %d of %d results",
                                                 n_zero, n_rets);
  const void* fn;
  int block, smem, occ, dev = 0, sms = 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    Kernel* k = find(id);
    if (!k) return fail(TM_EINVAL, "tallymap_b200: kernel id %lld is not registered in this process", (long long)id);
    if (n_args + n_rets != k->nbuf)
      return fail(TM_EINVAL, "tallymap_b200: kernel '%s' takes %d buffers, got %d + %d", k->name.c_str(), k->nbuf,
                  n_args, n_rets);
    int rc = ensure_loaded(*k);
    if (rc) return rc;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
    if ((rc = occupancy(*k, dev, &occ))) return rc;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail("cudaDeviceGetAttribute", e);
    fn = k->fn;
    block = k->block;
    smem = k->smem;
  }
  tmb::Params P;
  std::memset(&P, 0, sizeof(P));
  for (int i = 0; i < n_args + n_rets; ++i) {
    // an empty buffer may be null (no items: no kernel runs; an empty result is never written), and with flags
    // bit 3 the last argument (the item claim order) may be null
    const bool empty = i < n_args ? (n_items == 0 || ((flags & 8) && i == n_args - 1)) : ret_bytes[i - n_args] == 0;
    if (!bufs[i] && !empty) return fail(TM_EINVAL, "tallymap_b200: tm_launch: buffer %d is null", i);
    P.p[i] = bufs[i];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n_zero; ++i) {
    if (ret_bytes[i] == 0) continue;
    cudaError_t e = cudaMemsetAsync(bufs[n_args + i], 0, ret_bytes[i], st);
    if (e != cudaSuccess) {
      if (status) *status = (int32_t)e;
      return cuda_fail("cudaMemsetAsync", e);
    }
  }
  if (n_items == 0) return TM_OK;
  long long grid = (long long)sms * occ;
  const long long need = (n_items + block - 1) / block;
  if (grid > need && !(flags & 4)) grid = need;
  if (grid < 1) grid = 1;
  long long nn = n_items;
  void* args[] = {&P, &nn};
  cudaError_t e = cudaLaunchKernel(fn, dim3((unsigned)grid), dim3((unsigned)block), args, (size_t)smem, st);
  if (e != cudaSuccess) {
    if (status) *status = (int32_t)e;
    return cuda_fail("cudaLaunchKernel", e);
  }
  return TM_OK;
}

int tm_exact_combine(void* stream, const void* words, int32_t n_src, int32_t n_bins, float* out, int32_t* stats) {
  if (!words || !out || !stats || n_src < 1 || n_bins < 1)
    return fail(TM_EINVAL, "tallymap_b200: tm_exact_combine: bad arguments");
  const int blk = 128, grid = (n_bins + blk - 1) / blk;
  tmb::exact_combine_kernel<<<grid, blk, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const tmb::u64*>(words), n_src, n_bins, out, stats);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TM_OK : cuda_fail("exact_combine_kernel", e);
}

int tm_exact_scatter(void* stream, const float* vals, const int32_t* bins, int64_t n, int32_t n_bins, void* words,
                     float* out, int32_t* stats) {
  if ((n > 0 && (!vals || !bins)) || !words || !out || !stats || n < 0 || n_bins < 1)
    return fail(TM_EINVAL, "tallymap_b200: tm_exact_scatter: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t wbytes = ((size_t)n_bins * tmb::kExactWords + (n_bins + 1) / 2) * 8;
  cudaError_t e = cudaMemsetAsync(words, 0, wbytes, st);
  if (e != cudaSuccess) return cuda_fail("cudaMemsetAsync", e);
  if (n > 0) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    long long grid = (n + 255) / 256;
    if (grid > 8LL * sms) grid = 8LL * sms;
    tmb::exact_scatter_kernel<<<(unsigned)grid, 256, 0, st>>>(vals, bins, n, n_bins, static_cast<tmb::u64*>(words),
                                                              stats);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("exact_scatter_kernel", e);
  }
  tmb::exact_readout_kernel<<<(n_bins + 127) / 128, 128, 0, st>>>(static_cast<const tmb::u64*>(words), n_bins, out,
                                                                  stats);
  e = cudaGetLastError();
  return e == cudaSuccess ? TM_OK : cuda_fail("exact_readout_kernel", e);
}

// The exact scatter-add of tm_exact_scatter without a caller-provided scratch buffer and without allocating: for
// callers that cannot call cudaMalloc (see the header).  Clears the words it needs, then runs the same two kernels on
// the same stream.  Every device has its own copy of the fixed scratch, shared by every call on that device: calls on
// one device whose work can overlap on the GPU (other streams, other host threads) race on it and must be
// serialised by the caller; calls on different devices do not race.
int tm_exact_scatter_noalloc(void* stream, const float* vals, const int32_t* bins, int64_t n, int32_t n_bins,
                             float* out, int32_t* stats) {
  if ((n > 0 && (!vals || !bins)) || !out || !stats || n < 0 || n_bins < 1)
    return fail(TM_EINVAL, "tallymap_b200: tm_exact_scatter_noalloc: bad arguments");
  if (n_bins > TM_NOALLOC_MAX_BINS)
    return fail(TM_EINVAL, "tallymap_b200: tm_exact_scatter_noalloc: %d bins exceed its fixed scratch of %d bins; "
                "use tm_exact_scatter with a caller-provided scratch buffer", n_bins, TM_NOALLOC_MAX_BINS);
  void* words = nullptr;
  int rc = noalloc_words(&words);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t wbytes = ((size_t)n_bins * tmb::kExactWords + (n_bins + 1) / 2) * 8;
  cudaError_t e = cudaMemsetAsync(words, 0, wbytes, st);
  if (e != cudaSuccess) return cuda_fail("cudaMemsetAsync", e);
  if (n > 0) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    long long grid = (n + 255) / 256;
    if (grid > 8LL * sms) grid = 8LL * sms;
    tmb::exact_scatter_kernel<<<(unsigned)grid, 256, 0, st>>>(vals, bins, n, n_bins, static_cast<tmb::u64*>(words),
                                                              stats);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("exact_scatter_kernel", e);
  }
  tmb::exact_readout_kernel<<<(n_bins + 127) / 128, 128, 0, st>>>(static_cast<const tmb::u64*>(words), n_bins, out,
                                                                  stats);
  e = cudaGetLastError();
  return e == cudaSuccess ? TM_OK : cuda_fail("exact_readout_kernel", e);
}

int tm_tree_generations(void* stream, const void* records, int64_t n_records, int32_t record_bytes,
                        int32_t gen_offset, int32_t gen_bytes, int32_t n_gen, uint64_t* counts, uint64_t* cursor,
                        int32_t* lists) {
  if (n_records < 0 || n_records > INT32_MAX || (gen_bytes != 2 && gen_bytes != 4) || record_bytes < gen_bytes ||
      record_bytes % gen_bytes || gen_offset < 0 || gen_offset % gen_bytes || gen_offset + gen_bytes > record_bytes ||
      n_gen < 1 || n_gen > TM_TREE_MAX_GEN || !counts || !cursor || (n_records > 0 && (!records || !lists)))
    return fail(TM_EINVAL, "tallymap_b200: tm_tree_generations: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(counts, 0, (size_t)(n_gen + 1) * 8, st);
  if (e != cudaSuccess) return cuda_fail("cudaMemsetAsync", e);
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long grid = (n_records + 255) / 256;
  if (grid > 8LL * sms) grid = 8LL * sms;
  if (grid < 1) grid = 1;
  const unsigned char* rec = static_cast<const unsigned char*>(records);
  unsigned long long* const cnt = reinterpret_cast<unsigned long long*>(counts);
  unsigned long long* const cur = reinterpret_cast<unsigned long long*>(cursor);
  tmb::tree_hist_kernel<<<(unsigned)grid, 256, (size_t)(n_gen + 1) * 4, st>>>(rec, n_records, record_bytes,
                                                                               gen_offset, gen_bytes, n_gen, cnt);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("tree_hist_kernel", e);
  tmb::tree_scan_kernel<<<1, 32, 0, st>>>(cnt, n_gen, cur);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("tree_scan_kernel", e);
  if (n_records > 0) {
    const size_t smem = (size_t)((n_gen + 2) & ~1) * 4 + (size_t)n_gen * 8;
    if (smem > 48 * 1024) {
      e = cudaFuncSetAttribute(tmb::tree_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute", e);
    }
    tmb::tree_scatter_kernel<<<(unsigned)grid, 256, smem, st>>>(rec, n_records, record_bytes, gen_offset, gen_bytes,
                                                               n_gen, cur, lists);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("tree_scatter_kernel", e);
  }
  return TM_OK;
}

int tm_probe_threefry(void* stream, int32_t iters, uint32_t* out, int64_t out_len, int64_t* threads_used) {
  if (!out || iters < 1 || out_len < 128) return fail(TM_EINVAL, "tallymap_b200: tm_probe_threefry: bad arguments");
  int dev = 0, sms = 0, occ = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, tmb::probe_threefry_kernel, 128, 0);
  if (e != cudaSuccess) return cuda_fail("cudaOccupancyMaxActiveBlocksPerMultiprocessor", e);
  long long blocks = (long long)sms * (occ < 1 ? 1 : occ);
  if (blocks * 128 > out_len) blocks = out_len / 128;
  tmb::probe_threefry_kernel<<<(unsigned)blocks, 128, 0, static_cast<cudaStream_t>(stream)>>>((tmb::u32)iters, out);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("probe_threefry_kernel", e);
  if (threads_used) *threads_used = blocks * 128;
  return TM_OK;
}

int tm_probe_issue(void* stream, int32_t kind, int32_t iters, uint32_t* out, int64_t out_len,
                   int64_t* threads_used) {
  if (!out || iters < 1 || out_len < 128 || kind < 0 || kind > 5)
    return fail(TM_EINVAL, "tallymap_b200: tm_probe_issue: bad arguments");
  const void* fn = kind == 0 ? (const void*)tmb::probe_threefry_kernel
                 : kind == 1 ? (const void*)tmb::probe_fp32_kernel
                 : kind == 2 ? (const void*)tmb::probe_ode_kernel<0>
                 : kind == 3 ? (const void*)tmb::probe_ode_kernel<1>
                 : kind == 5 ? (const void*)tmb::probe_ode_kernel<2> : (const void*)tmb::probe_photon_kernel;
  int dev = 0, sms = 0, occ = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, 128, 0);
  if (e != cudaSuccess) return cuda_fail("cudaOccupancyMaxActiveBlocksPerMultiprocessor", e);
  long long blocks = (long long)sms * (occ < 1 ? 1 : occ);
  if (blocks * 128 > out_len) blocks = out_len / 128;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (kind == 0) tmb::probe_threefry_kernel<<<(unsigned)blocks, 128, 0, st>>>((tmb::u32)iters, out);
  else if (kind == 1) tmb::probe_fp32_kernel<<<(unsigned)blocks, 128, 0, st>>>((tmb::u32)iters, out);
  else if (kind == 2) tmb::probe_ode_kernel<0><<<(unsigned)blocks, 128, 0, st>>>((tmb::u32)iters, out);
  else if (kind == 3) tmb::probe_ode_kernel<1><<<(unsigned)blocks, 128, 0, st>>>((tmb::u32)iters, out);
  else if (kind == 5) tmb::probe_ode_kernel<2><<<(unsigned)blocks, 128, 0, st>>>((tmb::u32)iters, out);
  else tmb::probe_photon_kernel<<<(unsigned)blocks, 128, 0, st>>>((tmb::u32)iters, out);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("probe kernel", e);
  if (threads_used) *threads_used = blocks * 128;
  return TM_OK;
}

int tm_math_eval(void* stream, int32_t fn, const float* x, const float* y, float* out, int64_t n) {
  if (fn < 0 || fn >= tmm::kMathFns || n < 0 || (n > 0 && (!x || !out || ((fn == 4 || fn == 6 || fn == 21) && !y))))
    return fail(TM_EINVAL, "tallymap_b200: tm_math_eval: bad arguments");
  if (n == 0) return TM_OK;
  long long grid = (n + 255) / 256;
  if (grid > 4096) grid = 4096;
  tmb::math_eval_kernel<<<(unsigned)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(fn, x, y, out, n);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TM_OK : cuda_fail("math_eval_kernel", e);
}

int tm_check_status(const uint32_t* ctl_host) {
  if (!ctl_host) return fail(TM_EINVAL, "tallymap_b200: tm_check_status: null argument");
  const uint32_t w = ctl_host[tmb::kCtlError];
  if (w == 0u) return TM_OK;
  return fail(TM_EDEVICE, "tallymap_b200: device error word 0x%08x (bit 0: a device wait timed out; bit 1: a bounds "
              "check failed)", w);
}

}  // extern "C"
