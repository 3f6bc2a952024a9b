"""Hand-written sm_100a kernel templates, tried in order by the compiler."""
from .attention import AttentionTemplate
from .attention_small import AttentionSmallTemplate
from .common import TemplateMismatch
from .gemm import GemmTemplate
from .gemm_small import GemmSmallTemplate
from .pointwise import PointwiseTemplate
from .rows import RowsTemplate

TEMPLATES = [PointwiseTemplate, RowsTemplate, GemmTemplate, GemmSmallTemplate, AttentionTemplate,
             AttentionSmallTemplate]

__all__ = ["TEMPLATES", "TemplateMismatch", "PointwiseTemplate", "RowsTemplate", "GemmTemplate",
           "AttentionTemplate", "GemmSmallTemplate", "AttentionSmallTemplate"]
