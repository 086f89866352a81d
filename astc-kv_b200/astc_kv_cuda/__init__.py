"""astc_kv_cuda — B200 (sm_100a) decode-attention over ASTC-compressed KV caches.

Host-side mirror of the reference's ``astc_kv/codec.py`` whose decode, restore
and attention run in ``libakv_cuda.so`` (C ABI: include/akv_cuda.h).
"""
from ._lib import AkvError, lib
from .codec import (AstcEncoder, EncodedTensor, align, attention, attention_metrics, encode_tensor, errors,
                    fp16_ceil, fp16_floor)
from .ops import (Attention, DevicePlane, contiguous_astc_plane, contiguous_fp16_plane, decode_attention,
                  decode_blocks, decode_image, host_encode, init, paged_astc_plane, paged_fp16_plane,
                  random_blocks, restore_plane)

__version__ = "0.1.0"
