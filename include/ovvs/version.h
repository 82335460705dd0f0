#pragma once

/* The library reports the version of the ABI it implements (reference include/ovvs/version.h),
 * so bindings that gate on it keep working. */
#define OVVS_VERSION_MAJOR 0
#define OVVS_VERSION_MINOR 2
#define OVVS_VERSION_PATCH 0
#define OVVS_VERSION_STRING "0.2.0"
