"""Document pipeline: stages that pass, rewrite or drop ``{"text", "language", "slice",
"meta"}`` documents (reference: ``saint_llm_data/pipeline/*.py``)."""

from saint_llm_b200.data.pipeline.dedup import FingerprintDedup, MinHashDedup, minhash_signature, minhash_signatures
from saint_llm_b200.data.pipeline.filters import (
    DEFAULT_BLOCKED_DOMAINS,
    LengthQualityFilter,
    PerplexityFilter,
    PerplexityModel,
    QualityClassifier,
    QualityFilter,
    TranslationeseDetector,
    TranslationeseFilter,
    URLBlocklistFilter,
)
from saint_llm_b200.data.pipeline.stage import Document, Pipeline, Stage, TokenizeStage

__all__ = [
    "DEFAULT_BLOCKED_DOMAINS", "Document", "FingerprintDedup", "LengthQualityFilter", "MinHashDedup", "PerplexityFilter",
    "PerplexityModel", "Pipeline", "QualityClassifier", "QualityFilter", "Stage", "TokenizeStage",
    "TranslationeseDetector", "TranslationeseFilter", "URLBlocklistFilter", "minhash_signature", "minhash_signatures",
]
