// Shim for building the reference's thread-group sources out of tree as a CPU-only test oracle.
#pragma once
#define DTORCH_WITH_CUDA 0
