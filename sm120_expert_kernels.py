"""Drop-in module name of the reference extension.

Callers written against kkontosis/LayerStoRmExpertKernels do
`import sm120_expert_kernels as EK`; this module re-exports the B200 build
under that name with the same op names, arguments and defaults.
"""
from layerstormexpertkernels_b200 import *  # noqa: F401,F403
from layerstormexpertkernels_b200 import __all__  # noqa: F401
