// Status codes shared by device and host code: the public ones come from the C-ABI header.
#pragma once

#include "pa_b200.h"

// Wall-clock limit of every device-side wait (mbarrier phases): about one second.
#define PA_WAIT_LIMIT_NS 1000000000ull
