from genesis.model.hlrt import HLRT, HLRTConfig

__all__ = ["HLRT", "HLRTConfig"]
