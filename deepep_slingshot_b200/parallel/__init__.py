from .buffer import Buffer, Config, topk_idx_t
from .elastic import ElasticBuffer, EPHandle
from .reference import ReferenceBuffer
