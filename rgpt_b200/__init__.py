"""rgpt_b200: B200-native (sm_100a) kernels and host mirror of the rGPT training step.

Sub-modules:
  _lib       ctypes binding of librgpt_kernels.so (C ABI in include/rgpt.h)
  native     torch-tensor wrappers of each native entry point
  model      GPT / rGPT modules with the reference's Python API
  optimizer  Muon / DistMuon (NorMuon / DistNorMuon aliases)
  trainer    the training-step driver
"""
__version__ = "0.1.0"
