"""techjam-b200: B200-native (sm_100a) forward pass of the reference pre-LN encoder.

Public surface:
    techjam_b200.dispatcher.CANDIDATE          candidate spec (reference ``--candidate`` API)
    techjam_b200.dispatcher.DispatchingTransformer
    techjam_b200.model.B200Transformer          nn.Module with the reference parameter tree
    techjam_b200.ops                            kernel-level building blocks (torch tensors in/out)
    techjam_b200.build.build()                  compile libtj.so in-tree
"""

__version__ = "0.1.0"
