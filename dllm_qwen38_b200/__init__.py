"""dllm_qwen38_b200: Blackwell-native (sm_100a) block-diffusion training and inference for hybrid
Gated DeltaNet / gated-attention Qwen models.

The one modelling idea carried over from the reference (`__init__.py:1-7` of dllm-qwen38) is the
state fork: a recurrence cannot take an attention mask, so the clean stream is run once, its
fp32 recurrent state and short-conv tail are kept at every block boundary, and each noised block
starts from the clean-prefix state before it.
"""

__version__ = "0.1.0"
