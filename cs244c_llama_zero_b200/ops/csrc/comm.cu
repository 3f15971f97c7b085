// NVLink / NVSwitch collective kernels.
#include "comm.h"
