// Unity build of the LittleBit sm_100a library: every kernel file is one
// translation unit so device globals (the error word) have a single definition
// and no relocatable-device-code link step is needed.
#include <algorithm>

#include "capi.cu"
#include "pack.cu"
#include "linear.cu"
#include "chain.cu"
#include "wide.cu"
#include "misc.cu"
#include "attention.cu"
#include "lmhead.cu"
#include "program.cu"
#include "forward.cu"
