// Shim (oracle build): assertion and logging macros. Failures throw, so a broken oracle run surfaces as an
// error code from the harness instead of a silent result.
#pragma once
#include <sstream>
#include <stdexcept>
#include <string>

namespace dtorch {
struct ShimFatal {
    std::ostringstream os;
    bool fatal;
    explicit ShimFatal(bool f) : fatal(f) {}
    template <typename T>
    ShimFatal& operator<<(const T& v) { os << v; return *this; }
    ~ShimFatal() noexcept(false) {
        if (fatal) throw std::runtime_error("oracle fatal: " + os.str());
    }
};
}  // namespace dtorch

#define DAlwaysAssert(c) \
    do { if (!(c)) throw std::runtime_error(std::string("oracle assert failed: ") + #c); } while (0)
#define DAlwaysAssertMsg(c, m) \
    do { if (!(c)) throw std::runtime_error(std::string("oracle assert failed: ") + #c + " " + (m)); } while (0)
#define DDebugAssert(c) DAlwaysAssert(c)
#define DDebugAssertMsg(c, m) DAlwaysAssertMsg(c, m)
#define DLogFatal() ::dtorch::ShimFatal(true)
#define DLogError() ::dtorch::ShimFatal(false)
#define DLogInfo() ::dtorch::ShimFatal(false)
#define DUnimplemented() throw std::runtime_error("oracle: unimplemented path")
#define DUnsupportedImpl() throw std::runtime_error("oracle: unsupported path")
