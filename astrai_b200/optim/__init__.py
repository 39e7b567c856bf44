from astrai_b200.optim.fused import (
    FusedAdamW,
    Muon,
    MuonMix,
    clip_grad_norm_,
    is_muon_param,
    newton_schulz_batched,
    newton_schulz_reference,
)

__all__ = ["FusedAdamW", "Muon", "MuonMix", "clip_grad_norm_", "is_muon_param", "newton_schulz_batched",
           "newton_schulz_reference"]
