from astrai_b200.dataset.dataset import (
    BaseDataset,
    DatasetFactory,
    DPODataset,
    GRPODataset,
    SEQDataset,
    SFTDataset,
    dpo_collate_fn,
    dpo_processor,
    dpo_tokenize,
    grpo_collate_fn,
)
from astrai_b200.dataset.sampler import RDSampler
from astrai_b200.dataset.storage import (
    H5Store,
    JsonlSource,
    JsonlStore,
    MmapStore,
    Store,
    StoreFactory,
    detect_format,
)

__all__ = [
    "BaseDataset", "DatasetFactory", "DPODataset", "GRPODataset", "SEQDataset", "SFTDataset", "dpo_collate_fn",
    "dpo_processor", "dpo_tokenize", "grpo_collate_fn", "RDSampler", "H5Store", "JsonlSource", "JsonlStore",
    "MmapStore", "Store", "StoreFactory", "detect_format",
]
