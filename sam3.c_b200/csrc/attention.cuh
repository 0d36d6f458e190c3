// attention.cuh - fused attention launcher (attention.cu).
#pragma once
#include "sam3cu_internal.h"
