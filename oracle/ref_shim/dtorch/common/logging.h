// Shim (oracle build): logging macros live with the assertion macros.
#pragma once
#include "dtorch/common/debug.h"
