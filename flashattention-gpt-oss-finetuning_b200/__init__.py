"""B200 (sm_100a) causal sliding-window + sink-token + GQA attention, forward and backward.

Drop-in for the reference's ``flash_attention_gpt_oss`` entry points; the compute runs in the
C-ABI library ``lib/libswa_attn.so`` (``include/swa_attn.h``).
"""
from .flash_attention_gpt_oss import (FlashSWDAWithSink, FlashSWDAWithSinkLogits,
                                      flash_swda_with_sink, swa_backward,
                                      swa_forward)
from .varlen import FlashSWDAWithSinkVarlen, flash_swda_with_sink_varlen
from ._lib import SwaDeviceTimeout, SwaError, lib, lib_path

__all__ = ["FlashSWDAWithSink", "FlashSWDAWithSinkLogits", "flash_swda_with_sink", "swa_forward", "swa_backward",
           "FlashSWDAWithSinkVarlen", "flash_swda_with_sink_varlen",
           "SwaError", "SwaDeviceTimeout", "lib", "lib_path"]
