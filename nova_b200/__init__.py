"""nova_b200 -- B200-native (sm_100a) kernels for Nova's quantized decode hot path.

Drop-in modules mirroring the reference package ``nova`` (captain-wangrun-cn/Nova):

* ``nova_b200.kvquant``  quantize_int8 / dequantize_int8 (token axis, int8t64)
* ``nova_b200.kvattn``   int8_attn_decode, pack_int8_kv, tail_attend, KVInt8Cache

All compute goes through ``libnova_b200.so`` (C ABI in ``include/nova_b200.h``);
there is no CPU or Triton fallback.
"""

from ._lib import available, version

__all__ = ["available", "version"]
