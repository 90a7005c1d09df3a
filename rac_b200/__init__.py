"""rac_b200 -- the RAC rotation-accumulate hot path on NVIDIA B200 (sm_100a).

Layers:
  * librac_b200.so  -- CUDA kernels + the C ABI (include/rac.h, include/rac_b200.h)
  * rac_b200._lib   -- ctypes binding of that ABI
  * rac_b200.ext    -- torch-tensor front end (the reference's rac_cuda_ext surface)
  * rac_b200.rac_torch -- the reference's rac_torch module API
  * rac_b200.tp     -- N-column sharded matmul and the tensor-parallel Llama block
"""
__version__ = "0.1.0"
