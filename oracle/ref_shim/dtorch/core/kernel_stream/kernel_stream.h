// Shim (oracle build): nothing from the kernel-stream runtime is needed on the CPU path.
#pragma once
