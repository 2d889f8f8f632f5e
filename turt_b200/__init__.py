"""turt_b200 -- B200-native (sm_100a) backend for turt's GPU-resident GPT training step.

The compute path is libturt_cuda.so (hand-written CUDA, C ABI in include/turt_cuda.h).
This package is the Python host side: a ctypes binding, thin context/model handles, and a
mirror of the reference's GpuEngine / GpuTensor / GpuGPT / AdamW interfaces.
"""
