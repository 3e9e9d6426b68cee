from olympus.optim.muon import Muon
from olympus.optim.muon_adamw_hybrid import MuonAdamWHybrid
from olympus.optim.schedulers import WSDScheduler

__all__ = ["Muon", "MuonAdamWHybrid", "WSDScheduler"]
