// The XLA FFI binding of the launcher: the custom-call target a JAX install registers in place of the reference's
// "tallymap_cuda_launch" (tallymap/backends/kernel/shim.cc:241-250, bound from backends/kernel/__init__.py:173-176).
//
// It takes the reference's attribute set -- kernel_id, block, n_zero, flags, n_items -- and XLA's buffers (the
// operands, then the results), and hands them to tm_launch (include/tallymap_b200.h), which zeroes the first n_zero
// results and launches the registered kernel on XLA's stream.  `block` is the reference caller's thread-block size;
// here a kernel's block is fixed when it is registered (tm_register / tm_compile_register), so the handler checks
// that the two agree and refuses the call otherwise, instead of launching a different shape than the caller asked
// for.  Errors return ffi::Error with tm_last_error()'s text, as the reference's handler returns its own.
//
// The handler compiles only where XLA's FFI headers are on the include path (jax.ffi.include_dir(); the library's
// build adds it when JAX is importable).  tm_ffi_available() says whether this build has it.
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/tallymap_b200.h"

#if defined(__has_include)
#if __has_include("xla/ffi/api/ffi.h")
#define TM_HAVE_XLA_FFI 1
#endif
#endif

#ifdef TM_HAVE_XLA_FFI
#include <cuda_runtime.h>

#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

constexpr size_t kMaxBuffers = 64;   // the launch's parameter block holds at most 64 pointers (TM_MAXP)

ffi::Error tm_ffi_launch(cudaStream_t stream, ffi::RemainingArgs args, ffi::RemainingRets rets, int64_t kernel_id,
                         int32_t block, int32_t n_zero, int32_t flags, int64_t n_items) {
  const size_t na = args.size(), nr = rets.size();
  if (na + nr > kMaxBuffers)
    return ffi::Error(ffi::ErrorCode::kInvalidArgument,
                      "tallymap_b200: " + std::to_string(na + nr) + " buffers exceed the launch's 64");
  long long info[7];
  if (tm_kernel_info(kernel_id, info) != TM_OK)
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, tm_last_error());
  if (info[6] != (long long)block)
    return ffi::Error(ffi::ErrorCode::kInvalidArgument,
                      "tallymap_b200: the caller's block " + std::to_string(block) + " differs from kernel " +
                          std::to_string(kernel_id) + "'s registered block " + std::to_string(info[6]));
  void* bufs[kMaxBuffers];
  size_t ret_bytes[kMaxBuffers];
  for (size_t i = 0; i < na; ++i) {
    auto b = args.get<ffi::AnyBuffer>(i);
    if (!b.has_value()) return b.error();
    bufs[i] = b->untyped_data();
  }
  for (size_t i = 0; i < nr; ++i) {
    auto b = rets.get<ffi::AnyBuffer>(i);
    if (!b.has_value()) return b.error();
    bufs[na + i] = (*b)->untyped_data();
    ret_bytes[i] = (*b)->size_bytes();
  }
  int32_t status = 0;
  if (tm_launch(kernel_id, stream, bufs, (int32_t)na, (int32_t)nr, ret_bytes, n_zero, flags, n_items, &status) !=
      TM_OK)
    return ffi::Error(ffi::ErrorCode::kInternal, tm_last_error());
  return ffi::Error::Success();
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(TallymapB200Launch, tm_ffi_launch,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .RemainingArgs()
                                  .RemainingRets()
                                  .Attr<int64_t>("kernel_id")
                                  .Attr<int32_t>("block")
                                  .Attr<int32_t>("n_zero")
                                  .Attr<int32_t>("flags")
                                  .Attr<int64_t>("n_items"));

extern "C" int tm_ffi_available(void) { return 1; }

#else

extern "C" int tm_ffi_available(void) { return 0; }

#endif
