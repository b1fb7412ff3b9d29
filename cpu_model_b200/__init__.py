"""cpu_model_b200 -- B200-native (sm_100a) MX int8/int4 linear-layer hot path
of saoxdxd2/cpu_model behind a C-ABI (include/mxq.h, libmxq.so).

Importing the package does not touch the GPU; the operator mirror lives in
cpu_model_b200.mx and loads libmxq.so on first use.
"""
__version__ = "0.1.0"
