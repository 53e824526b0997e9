// Placement algebra of DTensor redistribution on a DeviceMesh: the semantics of the reference's
// dtorch/api/cpp/distributed_spec.{h,cc} and thread_group_manager.cc that the redistribute path depends on,
// restated for this library.
#pragma once

#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace dtb {

// Replicate, Partial (pending SUM over the mesh dim) or Shard(dim) -- dtorch/api/cpp/distributed_spec.h:94-169.
struct Placement {
    enum Kind { kReplicate = 0, kPartial = 1, kShard = 2 };
    Kind kind = kReplicate;
    int64_t dim = -1;       // tensor dim for kShard
    int64_t subSplit = -1;  // Shard(dim, subSplitCoordinates); -1 = plain shard

    static Placement Replicate() { return Placement{kReplicate, -1, -1}; }
    static Placement Partial() { return Placement{kPartial, -1, -1}; }
    static Placement Shard(int64_t d, int64_t sub = -1) { return Placement{kShard, d, sub}; }

    bool IsReplicate() const { return kind == kReplicate; }
    bool IsPartial() const { return kind == kPartial; }
    bool IsShard() const { return kind == kShard; }
    bool IsShard(int64_t d) const { return kind == kShard && dim == d; }
    bool HasSubSplit() const { return kind == kShard && subSplit != -1; }
    bool operator==(const Placement& o) const { return kind == o.kind && dim == o.dim && subSplit == o.subSplit; }
    bool operator!=(const Placement& o) const { return !(*this == o); }
    std::string ToString() const;
    // "R", "P", "S<dim>" (the reference's string form, python/dtorch/distributed_spec.py:167-176)
    static Placement Parse(const std::string& s);
};

using PlacementSeq = std::vector<Placement>;
std::string ToString(const PlacementSeq& p);

// Devices arranged row-major in `shape`; `ids` are global device ids.
struct DeviceMesh {
    std::vector<int64_t> shape;
    std::vector<int64_t> ids;
    size_t NumAxis() const { return shape.size(); }
    int64_t Count() const { return static_cast<int64_t>(ids.size()); }
    bool IsDistributed() const { return ids.size() > 1; }
};

// The first L % n ranks get floor(L/n) + 1 (Placement::GetShardSizeForAllRank, distributed_spec.cc:202-213).
std::vector<int64_t> ShardSizes(int64_t length, int64_t n);

// Mesh dims whose placement differs (PlacementSeq::GetDiffDims, distributed_spec.cc:316-325).
std::vector<size_t> GetDiffDims(const PlacementSeq& a, const PlacementSeq& b);

// Order of the per-mesh-dim conversions: every changed dim that is not Shard->Replicate first, in order, then
// the Shard->Replicate dims back to front (PlacementSeq::GetConvertOrder, distributed_spec.cc:327-343).
std::vector<size_t> GetConvertOrder(const PlacementSeq& src, const PlacementSeq& dst);

// Placements on mesh dims of size 1 become Replicate (PlacementSeq::ToReplicateWhenDimSizeEqualOne).
void ToReplicateWhenDimSizeEqualOne(PlacementSeq& p, const DeviceMesh& mesh);

// Shard(-k) -> Shard(ndim - k) (PlacementSeq::ShardDimToPositiveNumber).
void ShardDimToPositive(PlacementSeq& p, size_t ndim);

// Throws std::invalid_argument unless `placements` is valid for `shape` on `mesh`
// (DistributedSpec::CheckValid / CheckShapeValid, distributed_spec.cc:345-424).
void CheckValid(const std::vector<int64_t>& shape, const DeviceMesh& mesh, const PlacementSeq& placements);

// Devices of the thread group along mesh dim `dim` that contains `deviceId`: the devices that share every
// other mesh coordinate with it, in order of their coordinate along `dim` (ThreadGroupInfo,
// thread_group_manager.cc:20-70). The rank of a device is its index in this list.
std::vector<int64_t> GroupDeviceIds(const DeviceMesh& mesh, size_t dim, int64_t deviceId);

// Local shape of every device (DistributedSpec::ComputeLocalShape, distributed_spec.cc:539-587): mesh dims
// sharding the same tensor dim combine (row-major over those mesh dims); uneven splits follow ShardSizes.
std::map<int64_t, std::vector<int64_t>> ComputeLocalShapes(const std::vector<int64_t>& shape, const DeviceMesh& mesh,
                                                          const PlacementSeq& placements);

// Index of deviceId in ids (DistributedSpec::GetRankId).
int64_t RankOf(int64_t deviceId, const std::vector<int64_t>& ids);

}  // namespace dtb
