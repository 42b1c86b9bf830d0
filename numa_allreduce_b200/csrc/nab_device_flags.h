// Compile-time switches shared by host and device code.
#pragma once

// -DNAB_DEBUG_BOUNDS=1 compiles the device-side bounds checks in (see
// nab_device.cuh); release builds leave it 0.
#ifndef NAB_DEBUG_BOUNDS
#define NAB_DEBUG_BOUNDS 0
#endif
