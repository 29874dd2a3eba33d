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
    directory goes last on ``sys.path``, so nothing else is shadowed.  When
    this package's drop-in ``model.independent_memory`` already stands in
    ``sys.modules`` (under a ``model`` package with no files of its own), the
    reference's ``model`` directory is added to that package's path, so the
    import still finds the reference's file."""
    runtime = os.path.join(REF, 'runtime')
    if runtime not in sys.path:
        sys.path.append(runtime)
    pkg = sys.modules.get('model')
    model_dir = os.path.join(runtime, 'model')
    if pkg is not None and hasattr(pkg, '__path__') and model_dir not in list(pkg.__path__):
        pkg.__path__ = list(pkg.__path__) + [model_dir]
    import importlib
    return importlib.import_module('model.inference_kernels')
