"""gsdlq_b200 -- B200-native decode engine for GSD-LQ-packed decoders.

Host side of the engine.  The compute path is the CUDA library
``libgsdlq_cuda.so`` (sources in ``csrc/``, C-ABI in ``include/gsdlq.h``),
bound through ctypes in ``_lib``.  PyTorch is used only for device memory,
streams, CUDA graphs and torch.distributed.

Modules
  codebook  A2 lattice tables (the reference's _get_turbo_codebook)
  gsd2      .gsd2 container reader / writer and format validation
  packer    synthetic format-conformant packer (NumPy, and CUDA for big shapes)
  ops       thin wrappers from torch tensors to the C-ABI entry points
  model     GSDLQModel: the reference's load / forward_token / sample_token surface
  tp        tensor-parallel sharding of packed linears over NCCL
"""
__version__ = "0.1.0"
