// Host-side helpers shared by the extension's translation units.
#pragma once
#include <cstdint>

namespace bdion {

int* status_device_ptr();     // device view of the host-mapped status word
int status_read();            // host read, no device synchronisation
void status_clear();
uint64_t wait_limit_ns();     // limit for every bounded device wait
void set_wait_limit_ns(uint64_t ns);
void note_launch(int n = 1);  // count of this extension's kernel launches
uint64_t launch_count();

}  // namespace bdion
