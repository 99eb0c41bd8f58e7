// cuda_backend.h — the reference-side drop-in: splatx::KernelBackend on the B200 library.
//
// splatx-metal selects its kernels through one abstract class, splatx::KernelBackend
// (Sources/SplatXCore/include/splatx/KernelBackend.h:396-509), with make_metal_backend
// (MetalBackend.h:48-57) as the factory its Trainer, C training API and test runner call.
// make_cuda_backend is the CUDA counterpart: every KernelBackend method with the reference's
// host-vector semantics (inputs are host pointers, outputs fresh std::vectors, one synchronous
// call), std::invalid_argument for contract violations and std::runtime_error for device
// failures, and make_train_step_executor returning the resident executor
// (TrainStepExecutor, KernelBackend.h:386-392). Everything runs through the C-ABI of
// libsplatx_cuda.so (include/splatx_cuda.h); the adapter itself only stages host data into device
// buffers on its own CUDA stream.
//
// Built against the reference's headers (its include/ directory on the include path), as a
// maintainer would add it to the reference's build next to MetalBackend.cpp.
#pragma once

#include <memory>

#include "splatx/KernelBackend.h"

namespace splatx {

// The CUDA backend on device `device` (0-based CUDA ordinal). name() is "cuda(sm_100a)".
// Throws std::runtime_error when the device cannot be used.
std::unique_ptr<KernelBackend> make_cuda_backend(int device = 0);

}  // namespace splatx
