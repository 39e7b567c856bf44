from astrai_b200.preprocessing.builder import (
    BaseMaskBuilder,
    MaskBuilderFactory,
    MultiOutputMaskBuilder,
    SectionedMaskBuilder,
    SectionRenderer,
    SingleOutputMaskBuilder,
)
from astrai_b200.preprocessing.pipeline import (
    BFDPacking,
    BFDSplitPacking,
    BinWriter,
    H5Writer,
    PackingStrategyFactory,
    Pipeline,
    PositionIdStrategyFactory,
    SimplePacking,
    StoreWriterFactory,
    TokenizeTransform,
    filter_by_length,
    plan_bfd,
)

__all__ = [
    "BaseMaskBuilder", "MaskBuilderFactory", "MultiOutputMaskBuilder", "SectionedMaskBuilder", "SectionRenderer",
    "SingleOutputMaskBuilder", "BFDPacking", "BFDSplitPacking", "BinWriter", "H5Writer", "PackingStrategyFactory",
    "Pipeline", "PositionIdStrategyFactory", "SimplePacking", "StoreWriterFactory", "TokenizeTransform",
    "filter_by_length", "plan_bfd",
]
