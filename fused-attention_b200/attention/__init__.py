"""B200 (sm_100a) fused causal attention, drop-in for the reference's `attention` package.

Public modules (same paths and names as the reference project):
  attention.fused.fused.fused_attention                    causal MHA forward
  attention.gqa.fused_gqa.fused_gqa_attention              causal GQA/MQA forward
  attention.backward.fused_backward.fused_attention_autograd / FusedAttentionFn
  attention.fused.validation / attention.gqa.validation_gqa input contracts
All compute runs in hand-written sm_100a kernels (libfa_sm100.so) through a C ABI.
"""
