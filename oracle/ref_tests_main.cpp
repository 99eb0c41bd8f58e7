// Test runner of the reference's own kernel test translation units over the CUDA backend —
// TEST INFRASTRUCTURE.
//
// The reference's tests reach their backend through sxtest::shared_metal_backend()
// (Sources/SplatXTests/TestUtils.h:35-48), which calls splatx::make_metal_backend
// (MetalBackend.h:48-57). This file supplies both make_metal_backend overloads as stand-ins that
// return splatx::make_cuda_backend(0) (splatx-metal_b200/adapter/cuda_backend.h), so the unmodified
// test sources (Adam, ProjectionMetal, Sh, Isect, Sort, Scan, Raster, Ssim, Mcmc, McmcStrategy,
// Trainer) run against the B200 kernels. The fixtures come from $SPLATX_FIXTURE_DIR (TestPaths.h).
//
//   splatx_ref_tests [name ...]   runs the named tests (all when none are given) and prints one
//                                  "RESULT <PASS|FAIL> <name> <failed checks>" line per test;
//   splatx_ref_tests --list        prints the registered test names.
#include <cstdio>
#include <cstring>
#include <set>
#include <string>

#include <stdexcept>

#include "TestHarness.h"
#include "cuda_backend.h"
#include "splatx/ImageIO.h"
#include "splatx/MetalBackend.h"
#include "splatx_train_c.h"

namespace splatx {
std::unique_ptr<KernelBackend> make_metal_backend(void*, const MetalBackendDesc&) {
    return make_cuda_backend(0);
}
std::unique_ptr<KernelBackend> make_metal_backend(void*, const std::string&) {
    return make_cuda_backend(0);
}

// Apple ImageIO (ImageIO.cpp) and the C training API (TrainC.cpp) do not build on Linux and are
// not part of the kernel path: the few Trainer tests that decode PNG/JPEG files or run a whole
// training job through sx_train_run_args fail with this message instead.
[[noreturn]] static void not_here(const char* what) {
    throw std::runtime_error(std::string(what) + ": not available on this platform (Apple ImageIO / "
                             "the C training API are outside the CUDA backend)");
}
ImageF32 load_image_rgb_f32(const std::string&) { not_here("load_image_rgb_f32"); }
ImageF32 load_image_rgb_f32_downscaled(const std::string&, int) {
    not_here("load_image_rgb_f32_downscaled");
}
void save_png_rgb_f32(const ImageF32&, const std::string&) { not_here("save_png_rgb_f32"); }
}  // namespace splatx

extern "C" int32_t sx_train_run_args(const SxTrainArgs*, char* err_buf, int32_t err_buf_len) {
    if (err_buf && err_buf_len > 0)
        std::snprintf(err_buf, static_cast<size_t>(err_buf_len),
                      "sx_train_run_args: not available on this platform");
    return 1;
}

int main(int argc, char** argv) {
    auto& tests = sxtest::Registry::shared().tests;
    if (argc == 2 && std::strcmp(argv[1], "--list") == 0) {
        for (auto& t : tests) std::printf("%s\n", t.first.c_str());
        return 0;
    }
    if (argc > 1) {
        std::set<std::string> want(argv + 1, argv + argc);
        decltype(sxtest::Registry::shared().tests) kept;
        for (auto& t : tests)
            if (want.count(t.first)) kept.push_back(t);
        tests.swap(kept);
    }
    const int rc = sxtest::run_all([](const char* name, bool passed, int failed_checks) {
        std::printf("RESULT %s %s %d\n", passed ? "PASS" : "FAIL", name, failed_checks);
        std::fflush(stdout);
    });
    return rc;
}
