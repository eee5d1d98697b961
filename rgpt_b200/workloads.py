"""The benchmark workloads of the rGPT training step, by name.

Each entry is a model config in the reference's GPT(**cfg) vocabulary (conf/model/*.yaml keys)
plus the micro-batch B, sequence length T and gradient-accumulation count of one optimizer step:

  gpt-small   d_model 512, 8 heads (head dim 64), 8 layers, squared-ReLU FFN 512->2048->512,
              RMSNorm pre-norm, f_rmsnorm QK norm, RoPE base 10000, G1 gate, vocab 50304,
              seq 1024, micro-batch 16
  rgpt-small  2 layers applied n_recur=4 times, q_head adaptive halting (cal_halt_loss),
              detach_recur False, layer scale, otherwise as gpt-small, gradient accumulation 4
  gpt-350m    d_model 1024, 16 heads, 24 layers, FFN 4x squared ReLU, seq 1024, micro-batch 16
              per GPU (the data-parallel configuration)

Dropout is 0.1, the rate of every model config of the reference (conf/model/*.yaml). The optimizer
settings are conf/training/default.yaml's.

FFN_SWEEP is the fused linear+activation sweep (model/kernels.py:289-374): X [M, 512] ~ N(0, 1),
W1 [2048, 512] and W2 [2048, 512] ~ N(0, 0.02), upstream gradient ~ N(0, 1), M in FFN_SWEEP["M"].
MUON_SINGLE is the single-matrix optimizer step: W [2048, 512] ~ N(0, 0.02), G ~ N(0, 1) * 1e-2,
zero momentum, momentum 0.95, lr 0.02, 5 Newton-Schulz steps (optimizer.py:51-74), plus an AdamW step
on a 512-vector p ~ N(1, 0.01), g ~ N(0, 1e-3) (optimizer.py:80-116).
"""

COMMON = dict(detach_recur=False, max_seq_len=1024, dropout=0.1, norm_type="rmsnorm", norm_eps=1e-5,
              qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, pad_token_id=-100,
              tie_word_embeddings=False, vocab_size=50304)

WORKLOADS = {
    "gpt-small": dict(cfg=dict(COMMON, name="gpt", n_layers=8, n_recur=1, cal_halt_loss=False, n_heads=8,
                               d_model=512, use_layer_scale=False), B=16, T=1024, accum=1),
    "rgpt-small": dict(cfg=dict(COMMON, name="rgpt", n_layers=2, n_recur=4, cal_halt_loss=True, n_heads=8,
                                d_model=512, use_layer_scale=True), B=16, T=1024, accum=4),
    "gpt-350m": dict(cfg=dict(COMMON, name="gpt", n_layers=24, n_recur=1, cal_halt_loss=False, n_heads=16,
                              d_model=1024, use_layer_scale=False), B=16, T=1024, accum=1),
}

OPT = dict(lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)  # conf/training/default.yaml

FFN_SWEEP = dict(M=(8192, 16384, 32768, 65536), K=512, N=2048,
                 activations=("squared_relu", "gelu", "silu", "mish"), x_std=1.0, w_std=0.02)

MUON_SINGLE = dict(shape=(2048, 512), w_std=0.02, g_std=1e-2, momentum=0.95, lr=0.02, ns_steps=5, seed=0,
                   adam_n=512, adam_p_mean=1.0, adam_p_std=0.01, adam_g_std=1e-3)
