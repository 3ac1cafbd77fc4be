/* hvx_hf.h -- the corpus's fp16 element type.  The corpus spells binary16
 * `__fp16` (typedef __fp16 hvx_hf, e.g. kernels/expert/fp16_softmax/
 * kernel_api.h:3); x86 gcc spells it _Float16, so host builds pass
 * -D__fp16=_Float16.  CUDA code uses uint16_t bit patterns instead. */
#ifndef HEXCUDA_HVX_HF_H
#define HEXCUDA_HVX_HF_H
typedef __fp16 hvx_hf;
#endif
