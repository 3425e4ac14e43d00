"""B200-native (sm_100a) W4A16 GEMV, a drop-in for the operator API of Yu-TingLee/int4-GEMV-cuda.

Modules: ops (the compiled operators), quant (quantise / pack / unpack / dequantize),
reference (fp32 reference and tolerance rule), capi (ctypes front end of the C ABI),
sharded (the multi-GPU N-split / K-split stack).
"""
