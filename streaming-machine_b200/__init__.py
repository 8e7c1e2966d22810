"""base2-b200: a B200-native (sm_100a) engine for streaming-machine's integer-only ("all base 2") GPT-2 machine.

Submodules:
  convert  seeded fp32 weights and the fp32 -> base-2 conversion (restates the reference's base2_convert.py)
  engine   the host side of the CUDA engine: the base2.py-shaped interface over the C-ABI library libbase2cuda.so
  build    compiles csrc/ into libbase2cuda.so for sm_100a
"""
