// Single translation unit of libmote_cuda.so.  The components are separate
// files for reading; compiling them as one unit lets them share the
// per-device status word without relocatable device code.
#include "runtime.cu"
#include "q4_0_gemm_tcgen05.cu"
#include "q4_0_linear.cu"
#include "decoder_stack.cu"
#include "q8_0_linear.cu"
#include "kquant_linear.cu"
#include "layer_ops.cu"
#include "q4_0_codec.cu"
#include "comm.cu"
#include "dense_matmul.cu"
#include "attention.cu"
#include "attention_prefill.cu"
