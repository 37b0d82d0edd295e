#ifndef Q38_CONTRACTS_H
#define Q38_CONTRACTS_H

// The subset of the reference runtime's include/q38/contracts.h that the
// sampler headers need (contracts.h:11-17 fourcc/kContractVersion,
// contracts.h:19-26 DType), with identical definitions so that a runtime
// which already has its own contracts.h can use the sampler headers
// unchanged.  When integrating into that runtime, keep the runtime's
// contracts.h and do not copy this file.

#include <cstddef>
#include <cstdint>

namespace q38 {

constexpr std::uint16_t kContractVersion = 1;
constexpr std::uint32_t fourcc(char a, char b, char c, char d) {
    return static_cast<std::uint32_t>(static_cast<unsigned char>(a)) |
           (static_cast<std::uint32_t>(static_cast<unsigned char>(b)) << 8u) |
           (static_cast<std::uint32_t>(static_cast<unsigned char>(c)) << 16u) |
           (static_cast<std::uint32_t>(static_cast<unsigned char>(d)) << 24u);
}

enum class DType : std::uint16_t {
    kInvalid = 0,
    kBFloat16 = 1,
    kFloat32 = 2,
    kFloat16 = 3,
    kInt8 = 4,
    kFp8E4M3 = 5,
};

}  // namespace q38

#endif
