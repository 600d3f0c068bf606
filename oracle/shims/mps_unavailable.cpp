// Test-infrastructure shim: the reference's Metal backend (src/backends/mps_backend.mm)
// is Objective-C++ and cannot build off macOS. These two entry points
// (include/mini_mla/execution.hpp:67-69) report "unsupported" so that
// make_execution("cpu") links; nothing in the oracle asks for "mps".
#include "mini_mla/execution.hpp"

namespace mini_mla {
Result<std::unique_ptr<Execution>> make_mps_execution(Model&, Optimizer*, std::string_view,
                                                      const ExecutionOptions&) {
    return Result<std::unique_ptr<Execution>>::failure(ErrorCode::unsupported,
                                                       "Metal is unavailable in this build");
}
Result<Json> metal_device_info() {
    return Result<Json>::failure(ErrorCode::unsupported, "Metal is unavailable in this build");
}
} // namespace mini_mla
