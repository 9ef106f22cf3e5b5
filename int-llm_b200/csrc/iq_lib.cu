// iq_lib.cu -- single translation unit of libiq.so: device globals (the CORDIC
// tables) and kernels are shared by every component without relocatable code.
#include "iq_api.cu"
#include "iq_model.cu"
#include "iq_synth.cu"
#include "iq_noalloc.cu"
#include "iq_mgw.cu"
