from astrai_b200.dataset.sampler import RDSampler

__all__ = ["RDSampler"]
