"""B200-native decode-step RoPE + KV-cache append.

`decode_llm_kernel_b200.cuda` is the drop-in for the reference's `decode_kernels.cuda`
(same functions, signatures and errors); `decode_llm_kernel_b200.cuda.ops` holds the four ops.
The compute runs in hand-written sm_100a kernels behind the C ABI declared in
include/decode_rope.h (lib/libdecode_rope.so).
"""
__version__ = "0.1.0"
