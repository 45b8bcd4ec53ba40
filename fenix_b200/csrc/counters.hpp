// counters.hpp — launch counter shared by every kernel launch wrapper of the library.
#pragma once

namespace fxk {
void count_launch();
unsigned long long launch_count();
}  // namespace fxk
