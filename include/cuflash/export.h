#pragma once

// Symbol visibility for the cuflash B200 library.
//
// The library is built with -fvisibility=hidden; every public entry point is
// tagged CUFLASH_EXPORT.  Macro name and meaning follow the reference's
// include/cuflash/export.h:11-26 so that consumers compiled against the
// reference header keep working unchanged.

#ifndef CUFLASH_EXPORT_H
#define CUFLASH_EXPORT_H

#if defined(CUFLASH_BUILDING_SHARED)
#define CUFLASH_EXPORT __attribute__((visibility("default")))
#else
#define CUFLASH_EXPORT
#endif

#endif  // CUFLASH_EXPORT_H
