"""ACT-V verifier: encoder, scoring heads, negative samples, replay, distillation.

Same public names as ``genesis/verifier/__init__.py`` of the reference.
"""

from genesis.verifier.distillation import VerificationDistillation
from genesis.verifier.negative_generator import NegativeGenerator
from genesis.verifier.replay_buffer import ReplayBuffer
from genesis.verifier.verification_head import VerificationHead
from genesis.verifier.verifier_model import VerifierModel

__all__ = ["VerifierModel", "VerificationHead", "NegativeGenerator", "ReplayBuffer", "VerificationDistillation"]
