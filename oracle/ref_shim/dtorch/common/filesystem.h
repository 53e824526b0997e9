// Shim (oracle build): temp dir lookup (only reached on the NCCL branch, unused on CPU meshes).
#pragma once
#include <cstdlib>
#include <string>
namespace dtorch {
inline std::string GetTempDirectoryPath() {
    const char* t = std::getenv("TMPDIR");
    return t ? std::string(t) : std::string("/tmp");
}
}  // namespace dtorch
