// internal.h -- helpers shared between the library's translation units
// (defined in race_api.cu; not part of the C ABI).
#pragma once

namespace race {
int report_error(int code, const char *msg);  // sets race_last_error(), returns code
void clear_error();
void note_launch();  // bumps race_launch_counter()
}  // namespace race
