// make_execution with a "cuda" branch: the reference's factory (src/infer/inference.cpp:314-329)
// dispatches "cpu" and "mps"; a maintainer adding this backend adds one branch to it,
//
//     if (backend == "cuda")
//         return make_cuda_execution(m, o, 0);
//
// next to the "mps" one. The test build (oracle/Makefile, target cuda) leaves the reference's
// source untouched: it compiles src/infer/inference.cpp with its factory renamed to
// mm_reference_make_execution and links this translation unit, whose make_execution takes the
// "cuda" branch and hands every other backend to the reference's own factory. So the
// reference's unmodified trainer (train_model, src/train/trainer.cpp:479-482) runs its GRPO
// loop on this backend when TrainOptions::backend is "cuda".
#include "mini_mla/execution.hpp"

#include <cstdlib>

namespace mini_mla {

Result<std::unique_ptr<Execution>> make_cuda_execution(Model& model, Optimizer* optimizer, int device);
Result<std::unique_ptr<Execution>> mm_reference_make_execution(Model& m, Optimizer* o, std::string_view backend,
                                                               std::string_view precision,
                                                               const ExecutionOptions& options);

Result<std::unique_ptr<Execution>> make_execution(Model& m, Optimizer* o, std::string_view backend,
                                                  std::string_view precision, const ExecutionOptions& options) {
    if (backend != "cuda") return mm_reference_make_execution(m, o, backend, precision, options);
    auto valid = options.validate();
    if (!valid) return Result<std::unique_ptr<Execution>>::failure(valid.error());
    // fp16 tensor-core compute over fp32 master weights, whichever precision is named
    if (precision != "fp32" && precision != "fp16")
        return Result<std::unique_ptr<Execution>>::failure(ErrorCode::unsupported, "Select cuda/fp32|fp16");
    const char* dev = std::getenv("MM_CUDA_DEVICE");
    return make_cuda_execution(m, o, dev ? std::atoi(dev) : 0);
}

}  // namespace mini_mla
