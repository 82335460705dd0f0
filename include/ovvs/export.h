#pragma once

/* Symbol visibility for libovvs.
 *
 * The library is compiled with -fvisibility=hidden and -DOVVS_BUILD, so only functions marked
 * OVVS_API leave the shared object. Consumers include this header without OVVS_BUILD and get a
 * plain declaration (or dllimport on Windows). Same macro name and meaning as the reference's
 * include/ovvs/export.h:1-15, which consumers already depend on. */

#if defined(_WIN32) || defined(_WIN64)
#  if defined(OVVS_BUILD)
#    define OVVS_API __declspec(dllexport)
#  else
#    define OVVS_API __declspec(dllimport)
#  endif
#else
#  if defined(OVVS_BUILD)
#    define OVVS_API __attribute__((visibility("default")))
#  else
#    define OVVS_API
#  endif
#endif
