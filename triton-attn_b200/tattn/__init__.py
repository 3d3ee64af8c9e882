"""B200-native FlashAttention-2 (sm_100a CUDA behind a C ABI), drop-in for amaanmithani/triton-attn's
``tattn`` package (src/tattn/__init__.py:3-5)."""

from tattn.api import attention, cuda_available, triton_available

__all__ = ["attention", "cuda_available", "triton_available"]
