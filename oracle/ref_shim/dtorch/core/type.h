// Shim (oracle build): the subset of dtorch/core/type.h the thread-group sources use -- device kinds and
// ids, tensor shapes, and the shard-size rule of Placement::GetShardSizeForAllRank
// (dtorch/api/cpp/distributed_spec.cc:202-213: the first L % n ranks get floor(L/n) + 1).
#pragma once
#include <cstdint>
#include <vector>

#include <torch/torch.h>

#include "dtorch/common/debug.h"
#include "dtorch/common/utilities.h"

namespace dtorch {
namespace api {
namespace cpp {

enum class DeviceKind { kCpu = 0, kGpu = 1 };

struct Device {
    DeviceKind deviceKind = DeviceKind::kCpu;
    int64_t deviceId = 0;
    Device() = default;
    explicit Device(DeviceKind k, int64_t id = 0) : deviceKind(k), deviceId(id) {}
    bool operator==(const Device& o) const { return deviceKind == o.deviceKind && deviceId == o.deviceId; }
    bool operator!=(const Device& o) const { return !(*this == o); }
};

class Shape {
public:
    Shape() = default;
    explicit Shape(std::vector<int64_t> d) : mDims(std::move(d)) {}
    size_t NumAxis() const { return mDims.size(); }
    int64_t& operator[](size_t i) { return mDims[i]; }
    int64_t operator[](size_t i) const { return mDims[i]; }
    const std::vector<int64_t>& Vec() const { return mDims; }
    bool operator==(const Shape& o) const { return mDims == o.mDims; }

private:
    std::vector<int64_t> mDims;
};

class Placement {
public:
    static std::vector<int64_t> GetShardSizeForAllRank(int64_t shapeSize, int64_t numShard) {
        DDebugAssert(shapeSize >= numShard);  // active in the reference's default build (DTORCH_DEBUG ON)
        std::vector<int64_t> out(static_cast<size_t>(numShard), shapeSize / numShard);
        for (int64_t i = 0; i < shapeSize % numShard; ++i) out[static_cast<size_t>(i)] += 1;
        return out;
    }
};

}  // namespace cpp
}  // namespace api

namespace core {
using api::cpp::Device;
using api::cpp::DeviceKind;
using api::cpp::Placement;
using api::cpp::Shape;
class Operand;
}  // namespace core
}  // namespace dtorch
