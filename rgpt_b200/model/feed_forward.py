"""FeedForward (model/feed_forward.py:17-37): fc1 [4d, d], fc2 [d, 4d], no bias."""
import torch.nn as nn

from .kernels import FusedLinearActivationFunction


class FeedForward(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.act_type = config.activation_type
        self.fc1 = nn.Linear(config.d_model, config.d_model * 4, bias=False)
        self.fc2 = nn.Linear(config.d_model * 4, config.d_model, bias=False)

    def forward(self, x):
        bsz, seq_len, d_model = x.shape
        out = FusedLinearActivationFunction.apply(x.reshape(-1, d_model), self.fc1.weight, self.fc2.weight.t(),
                                                  self.act_type)
        return out.view(bsz, -1, d_model)
