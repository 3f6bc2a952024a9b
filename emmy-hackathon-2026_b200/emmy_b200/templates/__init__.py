"""Hand-written sm_100a kernel templates, tried in order by the compiler."""
from .attention import AttentionTemplate
from .common import TemplateMismatch
from .gemm import GemmTemplate
from .pointwise import PointwiseTemplate
from .rows import RowsTemplate

TEMPLATES = [PointwiseTemplate, RowsTemplate, GemmTemplate, AttentionTemplate]

__all__ = ["TEMPLATES", "TemplateMismatch", "PointwiseTemplate", "RowsTemplate", "GemmTemplate",
           "AttentionTemplate"]
