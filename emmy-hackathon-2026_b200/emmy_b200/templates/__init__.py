"""Hand-written sm_100a kernel templates, tried in order by the compiler."""
from .common import TemplateMismatch
from .pointwise import PointwiseTemplate
from .rows import RowsTemplate

TEMPLATES = [PointwiseTemplate, RowsTemplate]

__all__ = ["TEMPLATES", "TemplateMismatch", "PointwiseTemplate", "RowsTemplate"]
