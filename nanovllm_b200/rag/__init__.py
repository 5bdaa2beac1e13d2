"""Retrieval: corpus loading and chunking, BM25, dense and hybrid indexes, ``RagSession``, ``RagFactory``."""
from .corpus import CorpusLoader, RagLoadOptions, RagResource, RagTuner, TextChunk
from .dense import DenseRagIndex, HybridRagIndex
from .factory import RagBuilder, RagFactory
from .lexical import PreparedRag, RagHit, RagIndex
from .session import RagSession, format_user_message

__all__ = ["CorpusLoader", "RagLoadOptions", "RagResource", "RagTuner", "TextChunk", "DenseRagIndex",
           "HybridRagIndex", "RagBuilder", "RagFactory", "PreparedRag", "RagHit", "RagIndex", "RagSession",
           "format_user_message"]
