"""B200-native (sm_100a) Q8_0 hot path of synthesize.cpp.

Import through __graft_entry__.load_package() or any loader that registers
this directory as the package ``synthesize_cpp_b200`` (the directory name
contains a dot, so a plain ``import`` cannot name it).

Submodules:
  q8     -- mul_mat / get_rows / quantize_chunk / quantize_rows / dequantize_rows
  chain  -- the talker-shaped decode step (DecodeChain)
  build  -- the nvcc / g++ recipe for the in-tree libraries
"""
from . import build  # noqa: F401
from ._abi import B200Q8Error, header_symbols, lib  # noqa: F401
