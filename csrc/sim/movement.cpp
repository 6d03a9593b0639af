// movement.cpp — host-side pieces of the movement module (the tick itself is
// header-only in movement.hpp, compiled for host and device).
#include "movement.hpp"

namespace surf {
namespace {
struct HostStuckTable {
  float v[54][3];
  HostStuckTable() {
    for (int i = 0; i < 54; ++i)
      for (int k = 0; k < 3; ++k) v[i][k] = mv::stuck_offset(i, k);
  }
};
const HostStuckTable kHostStuck;
}  // namespace

const float (*stuck_offsets())[3] { return kHostStuck.v; }

}  // namespace surf
