"""B200-native (sm_100a) Neural Cellular Automaton test-time rollout.

Drop-in for the rollout path of JorisViaudQuantAI/NCAs: `ncas_b200.rollout.rollout` has the
signature and result of nca.rollout.rollout, `ncas_b200.model.NCA` the parameter layout and
rollout-path methods of nca.model.NCA, and `ncas_b200.engine.B200RolloutBlocks` the call of
nca.engine.inference.UniformRolloutBlocks.  Compute runs in libnca_b200.so (CUDA, tcgen05),
loaded through ctypes from ncas_b200/_lib; there is no CPU fallback.
"""

__version__ = "0.1.0"
