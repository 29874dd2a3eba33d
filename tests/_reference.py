"""Access to the reference project installed under ``baseline/_ref`` (the
driver's one offline install of RocoreMatrix/YANchor, which travels with the
repository to the GPU box).  Tests that need the reference's own code import
it through these helpers; nothing in the package does."""
import os
import sys

from conftest import ROOT

REF = os.path.join(ROOT, 'baseline', '_ref')


def available():
    return os.path.exists(os.path.join(REF, 'modeling_yanchor.py'))


def inference_kernels():
    """The reference's ``model.inference_kernels`` (needs only torch).  Its
    directory goes last on ``sys.path``, so nothing else is shadowed."""
    runtime = os.path.join(REF, 'runtime')
    if runtime not in sys.path:
        sys.path.append(runtime)
    import importlib
    return importlib.import_module('model.inference_kernels')
