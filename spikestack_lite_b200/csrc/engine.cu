// Single translation unit of libspk_b200.so: the kernels share device state
// (the device error word) and inline helpers without relocatable device code.
#include "runtime.cu"
#include "csr.cu"
#include "spmm_csr.cu"
#include "spike_linear_tc.cu"
#include "spike_linear_tf32.cu"
#include "spike_linear_wt.cu"
#include "spike_linear.cu"
#include "attention.cu"
#include "attention_tc.cu"
#include "gsmc.cu"
#include "layernorm.cu"
#include "csr_noalloc.cu"
