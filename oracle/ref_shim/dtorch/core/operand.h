// Shim (oracle build): Operand as the thread-group sources see it -- per-device local shapes of a DTensor
// and whether the split is even (the reference's Operand::GetLocalShape / IsLocalShapeEventSplit).
#pragma once
#include <map>

#include "dtorch/core/type.h"

namespace dtorch {
namespace core {
class Operand {
public:
    Operand(std::map<int64_t, Shape> shapes, bool even) : mShapes(std::move(shapes)), mEven(even) {}
    Shape GetLocalShape(int64_t deviceId) const { return mShapes.at(deviceId); }
    bool IsLocalShapeEventSplit() const { return mEven; }

private:
    std::map<int64_t, Shape> mShapes;
    bool mEven;
};
}  // namespace core
}  // namespace dtorch
