// driver.cuh -- access to the driver-call table (include/ncz_driver.h) for the
// flash-attention and GEMM translation units, and the hooks through which
// ncz_set_driver releases and resets their per-device state.
#pragma once
#include "ncz_driver.h"

namespace ncz {

// The table in use: the CUDA runtime unless ncz_set_driver installed another.
const ncz_driver_table &drv();

// Flash translation unit: releases the split-KV pools and the host-pipeline
// streams and events through drv() (first error as an ncz_status), then drops
// every cached per-device value and the initialisation.
int release_flash_objects();
void reset_flash_caches();
const char *flash_kernel_label(const void *kernel);

// GEMM translation unit: drops its kernel-attribute and SM-count caches.
void reset_mma_caches();
const char *mma_kernel_label(const void *kernel);

}  // namespace ncz
