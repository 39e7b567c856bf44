"""astrai_b200: a Blackwell-native Transformer training and inference framework."""

__version__ = "0.1.0"
