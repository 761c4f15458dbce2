"""B200-native expert-parallel communication library (NVLink 5 / NVSwitch, sm_100a).

Capabilities and public API of the DeepEP v2 stack driven by swiss-ai/DeepEP_Slingshot, re-designed
for one 8xB200 box: `Buffer` (v1 API: layout, normal dispatch/combine, low-latency dispatch/combine
with receive hooks), `ElasticBuffer` / `EPHandle` (v2 API), `EventOverlap`, `Config`, plus the
pure-torch `ReferenceBuffer` oracle that also runs on CPU/gloo ranks.
"""
import torch

from ._ext import load_ext
from .parallel import Buffer, Config, ElasticBuffer, EPHandle, ReferenceBuffer, topk_idx_t
from .utils.envs import get_logical_domain_size, get_physical_domain_size
from .utils.event import EventOverlap

__version__ = '0.1.0'


def __getattr__(name):
    if name == 'EventHandle':
        from ._ext import require_ext
        return require_ext().EventHandle
    raise AttributeError(name)
