"""Op wrappers: CUDA tensors go to the sm_100a kernels in `_C`; CPU tensors run the fp32 torch oracle of the same op."""
