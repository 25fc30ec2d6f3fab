// Host-side fault injection (si_fault_inject): the allocation and file-read
// sites below ask fault_fire() before the real call and, when it fires, fail
// as that call would. Process-wide; each armed site fires once.
#pragma once
#include <cstdint>

namespace si {
constexpr uint32_t SI_FAULT_SITES = 4;  // 0 (none) + the three SI_FAULT_* sites
bool fault_fire(uint32_t site);
}  // namespace si
