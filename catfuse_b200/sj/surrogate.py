"""Surrogate-gradient placeholders.  Inference only: the forward is the
Heaviside step; the classes exist so model builders accept them."""
import torch


class SurrogateFunctionBase:
    def __init__(self, alpha=4.0, spiking=True):
        self.alpha = alpha
        self.spiking = spiking

    def __call__(self, x):
        return (x >= 0).to(x.dtype)


class Sigmoid(SurrogateFunctionBase):
    pass


class ATan(SurrogateFunctionBase):
    pass
