// Placement algebra (see placement.h for the reference functions each one restates).
#include "placement.h"

#include <algorithm>
#include <set>
#include <sstream>

namespace dtb {

std::string Placement::ToString() const {
    if (kind == kReplicate) return "R";
    if (kind == kPartial) return "P";
    if (subSplit == -1) return "S" + std::to_string(dim);
    return "S" + std::to_string(dim) + "/" + std::to_string(subSplit);
}

Placement Placement::Parse(const std::string& s) {
    if (s == "R") return Replicate();
    if (s == "P") return Partial();
    if (s.size() >= 2 && s[0] == 'S') {
        const auto slash = s.find('/');
        const int64_t d = std::stoll(s.substr(1, slash == std::string::npos ? std::string::npos : slash - 1));
        const int64_t sub = slash == std::string::npos ? -1 : std::stoll(s.substr(slash + 1));
        return Shard(d, sub);
    }
    throw std::invalid_argument("bad placement string: " + s);
}

std::string ToString(const PlacementSeq& p) {
    std::ostringstream os;
    os << "[";
    for (size_t i = 0; i < p.size(); ++i) os << (i ? ", " : "") << p[i].ToString();
    os << "]";
    return os.str();
}

std::vector<int64_t> ShardSizes(int64_t length, int64_t n) {
    if (n <= 0) throw std::invalid_argument("ShardSizes: n must be positive");
    std::vector<int64_t> out(static_cast<size_t>(n), length / n);
    for (int64_t i = 0; i < length % n; ++i) out[static_cast<size_t>(i)] += 1;
    return out;
}

std::vector<size_t> GetDiffDims(const PlacementSeq& a, const PlacementSeq& b) {
    if (a.size() != b.size()) throw std::invalid_argument("placement sequences differ in length");
    std::vector<size_t> out;
    for (size_t i = 0; i < a.size(); ++i)
        if (a[i] != b[i]) out.push_back(i);
    return out;
}

std::vector<size_t> GetConvertOrder(const PlacementSeq& src, const PlacementSeq& dst) {
    std::vector<size_t> front, shard_to_rep;
    for (size_t i = 0; i < src.size(); ++i) {
        if (src[i].IsShard() && dst[i].IsReplicate()) {
            shard_to_rep.push_back(i);
        } else if (src[i] != dst[i]) {
            front.push_back(i);
        }
    }
    front.insert(front.end(), shard_to_rep.rbegin(), shard_to_rep.rend());
    return front;
}

void ToReplicateWhenDimSizeEqualOne(PlacementSeq& p, const DeviceMesh& mesh) {
    if (p.size() != mesh.NumAxis()) throw std::invalid_argument("placements and mesh differ in rank");
    for (size_t i = 0; i < p.size(); ++i)
        if (mesh.shape[i] == 1) p[i] = Placement::Replicate();
}

void ShardDimToPositive(PlacementSeq& p, size_t ndim) {
    const int64_t n = static_cast<int64_t>(ndim);
    for (auto& q : p)
        if (q.IsShard() && q.dim < 0 && q.dim >= -n) q = Placement::Shard(q.dim + n, q.subSplit);
}

namespace {

struct ShardInfo {
    int64_t shardSize = 1;
    std::vector<size_t> meshDims;  // increasing
};

std::map<int64_t, ShardInfo> GetShardInfo(const DeviceMesh& mesh, const PlacementSeq& p) {
    std::map<int64_t, ShardInfo> out;
    for (size_t i = 0; i < p.size(); ++i) {
        if (!p[i].IsShard()) continue;
        ShardInfo& s = out[p[i].dim];
        s.shardSize *= mesh.shape[i];
        s.meshDims.push_back(i);
    }
    return out;
}

std::vector<int64_t> Coordinates(const DeviceMesh& mesh, size_t linear) {
    std::vector<int64_t> c(mesh.NumAxis());
    for (size_t d = mesh.NumAxis(); d-- > 0;) {
        c[d] = static_cast<int64_t>(linear) % mesh.shape[d];
        linear /= static_cast<size_t>(mesh.shape[d]);
    }
    return c;
}

}  // namespace

void CheckValid(const std::vector<int64_t>& shape, const DeviceMesh& mesh, const PlacementSeq& p) {
    if (p.empty()) throw std::invalid_argument("empty placement sequence");
    if (p.size() != mesh.NumAxis())
        throw std::invalid_argument("DeviceMesh and placements differ in size: " + std::to_string(mesh.NumAxis()) +
                                    " vs " + std::to_string(p.size()));
    int64_t count = 1;
    for (auto s : mesh.shape) count *= s;
    if (count != mesh.Count()) throw std::invalid_argument("mesh shape does not match its device count");
    if (mesh.Count() == 1 && !p[0].IsReplicate())
        throw std::invalid_argument("DeviceMesh has one device, but the placement is not Replicate");
    if (std::set<int64_t>(mesh.ids.begin(), mesh.ids.end()).size() != mesh.ids.size())
        throw std::invalid_argument("DeviceMesh has duplicate device ids");
    for (size_t i = 0; i < p.size(); ++i) {
        if (!p[i].IsShard()) continue;
        if (p[i].dim < 0) throw std::invalid_argument("shard dim less than zero: " + std::to_string(p[i].dim));
        if (p[i].dim >= static_cast<int64_t>(shape.size()))
            throw std::invalid_argument("shard dim larger than the tensor rank: " + std::to_string(p[i].dim));
        if (mesh.shape[i] < 2) throw std::invalid_argument("shard size less than 2");
        if (p[i].subSplit != -1 && p[i].subSplit < 0)
            throw std::invalid_argument("subSplitCoordinates must be -1 or >= 0");
    }
    for (const auto& kv : GetShardInfo(mesh, p)) {
        if (shape[static_cast<size_t>(kv.first)] < kv.second.shardSize)
            throw std::invalid_argument("cannot shard dim " + std::to_string(kv.first) + " of size " +
                                        std::to_string(shape[static_cast<size_t>(kv.first)]) + " into " +
                                        std::to_string(kv.second.shardSize) + " shards");
    }
}

std::vector<int64_t> GroupDeviceIds(const DeviceMesh& mesh, size_t dim, int64_t deviceId) {
    if (dim >= mesh.NumAxis()) throw std::invalid_argument("mesh dim out of range");
    if (mesh.NumAxis() == 1) return mesh.ids;
    int64_t left = 1, right = 1;
    const int64_t mid = mesh.shape[dim];
    for (size_t i = 0; i < dim; ++i) left *= mesh.shape[i];
    for (size_t i = dim + 1; i < mesh.NumAxis(); ++i) right *= mesh.shape[i];
    for (int64_t l = 0; l < left; ++l) {
        for (int64_t r = 0; r < right; ++r) {
            for (int64_t m = 0; m < mid; ++m) {
                if (mesh.ids[static_cast<size_t>((l * mid + m) * right + r)] != deviceId) continue;
                std::vector<int64_t> out;
                for (int64_t k = 0; k < mid; ++k) out.push_back(mesh.ids[static_cast<size_t>((l * mid + k) * right + r)]);
                return out;
            }
        }
    }
    throw std::invalid_argument("device " + std::to_string(deviceId) + " is not in the mesh");
}

std::map<int64_t, std::vector<int64_t>> ComputeLocalShapes(const std::vector<int64_t>& shape, const DeviceMesh& mesh,
                                                          const PlacementSeq& p) {
    std::vector<int64_t> even = shape;
    const auto infos = GetShardInfo(mesh, p);
    for (const auto& kv : infos) {
        const size_t d = static_cast<size_t>(kv.first);
        if (shape[d] % kv.second.shardSize == 0) even[d] = shape[d] / kv.second.shardSize;
    }
    std::map<int64_t, std::vector<int64_t>> out;
    for (auto id : mesh.ids) out[id] = even;
    for (const auto& kv : infos) {
        const size_t d = static_cast<size_t>(kv.first);
        // sub-split Shard(d, s) on one mesh dim: piece i = piece i of the first s + 1 rows plus piece i of the
        // rest (ReplicateToShard, thread_group.cc:258-276; DistributedScather, distributed_scather_and_gather.cc:61-80)
        int64_t sub = -1;
        for (auto md : kv.second.meshDims)
            if (p[md].HasSubSplit()) sub = p[md].subSplit;
        std::vector<int64_t> split;
        if (sub >= 0) {
            if (kv.second.meshDims.size() != 1)
                throw std::invalid_argument("a sub-split shard dim must be sharded by one mesh dim");
            if (sub <= 0 || sub >= shape[d]) throw std::invalid_argument("invalid subSplitCoordinates");
            const auto front = ShardSizes(sub + 1, kv.second.shardSize);
            const auto back = ShardSizes(shape[d] - sub - 1, kv.second.shardSize);
            for (size_t i = 0; i < front.size(); ++i) split.push_back(front[i] + back[i]);
        } else {
            if (shape[d] % kv.second.shardSize == 0) continue;
            split = ShardSizes(shape[d], kv.second.shardSize);
        }
        for (size_t idx = 0; idx < mesh.ids.size(); ++idx) {
            const auto c = Coordinates(mesh, idx);
            int64_t sel = 0;  // row-major index over the selected mesh dims
            for (auto md : kv.second.meshDims) sel = sel * mesh.shape[md] + c[md];
            out[mesh.ids[idx]][d] = split[static_cast<size_t>(sel)];
        }
    }
    return out;
}

int64_t RankOf(int64_t deviceId, const std::vector<int64_t>& ids) {
    for (size_t i = 0; i < ids.size(); ++i)
        if (ids[i] == deviceId) return static_cast<int64_t>(i);
    throw std::invalid_argument("device " + std::to_string(deviceId) + " not in the device list");
}

}  // namespace dtb
