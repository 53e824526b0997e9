// Shim (oracle build): communication timeout knob (DTORCH_COMM_TIMEOUT_SECOND, default 600 s).
#pragma once
#include <cstdint>
#include <cstdlib>
namespace dtorch {
namespace core {
class GlobalOption {
public:
    static GlobalOption& GetSingleton() {
        static GlobalOption g;
        return g;
    }
    int64_t GetCommTimeoutSecond() const { return mTimeout; }

private:
    GlobalOption() {
        const char* s = std::getenv("DTORCH_COMM_TIMEOUT_SECOND");
        mTimeout = (s && std::atoll(s) > 0) ? std::atoll(s) : 600;
    }
    int64_t mTimeout;
};
}  // namespace core
}  // namespace dtorch
