// Test infrastructure: bf16 storage types for the host build of the
// library's fp32 launchers (defined by tests/simt_host.h).
#pragma once

#include "simt_host.h"
