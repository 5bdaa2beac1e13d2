"""``LlmModelFactory``: path -> ``LlmModel`` over the three checkpoint containers.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/LlmModelFactory.java:94-895 (load
dispatch: a ``.gguf`` file -> GGUF causal (qwen3, lfm2) or embedding (bert); a Hugging Face folder ->
safetensors when present, else ONNX; tokenizer from tokenizer.json -> tokenizer.model -> GGUF metadata;
``ModelSupport.require`` before any payload is read; options map; Builder) and the architecture processors'
bind / fill steps (llmarch/*).  Weights are returned as a name -> tensor map in the names each model graph
consumes: Hugging Face names for qwen3 / llama / gemma3 / gemma4 (GGUF qwen3 tensors renamed), GGUF names for lfm2
and bert (ONNX BERT names mapped onto them).  GGUF blocks are dequantised at load (on the GPU when one is present).
"""
from __future__ import annotations

import os
import re
from typing import Dict, Optional

import torch

from ..config import HfConfig
from ..exceptions import ModelLoadException, UnsupportedModelException
from ..ops.quant import GgufPacked, fused_supported
from ..loaders import model_support as MS
from ..loaders.gguf import GgufFile
from ..loaders.gguf_configs import hf_config_from_gguf, hf_name_for_qwen3
from ..tokenizer.tokenizer import Tokenizer
from .model import LlmModel

OPTION_THINK_TAGS = "think_tags"
OPTION_CHAT_SPECIALS = "chat_specials"
OPTION_LISTENER = "listener"  # an LlmListener that receives load progress events
OPTION_UNPACK = "unpack_parameters"  # expand packed weights (GGUF blocks, QAT integers) to bf16 at load


def _is_gguf(path: str) -> bool:
    if not os.path.isfile(path):
        return False
    with open(path, "rb") as f:
        return f.read(4) == b"GGUF"


def _load_device(device) -> torch.device:
    if device is not None:
        return torch.device(device)
    return torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")


class LlmModelFactory:
    @staticmethod
    def catalog(path):
        """Bind ``path`` from its headers only (architecture, config, tensor names / shapes / types), without
        reading any tensor payload; ``.require_complete()`` checks it against the architecture's schema."""
        from ..loaders.catalog import ContainerCatalog
        return ContainerCatalog.bind(path)

    @staticmethod
    def make(path, options: Optional[dict] = None, device=None, dtype=torch.bfloat16) -> LlmModel:
        """``path``: a model folder, a .gguf file, or a ``ModelFileSource`` (api.sources)."""
        from .sources import ModelFileSource
        if isinstance(path, ModelFileSource):
            src = path
            try:
                return LlmModelFactory.make(src.local_path(), options, device, dtype)
            finally:
                src.close()
        path = os.fspath(path)
        if _is_gguf(path) or path.lower().endswith(".gguf"):
            return _load_gguf(path, options, _load_device(device), dtype)
        if os.path.isdir(path):
            return _load_hf_folder(path, options, _load_device(device), dtype)
        raise ModelLoadException(f"model path not found or not a GGUF file / model folder: {path}")

    class Builder:
        def __init__(self):
            self._path = None
            self._options = {}
            self._device = None

        def path(self, p):
            self._path = p
            return self

        def option(self, k, v):
            self._options[k] = v
            return self

        def think_tags(self, tags):
            self._options[OPTION_THINK_TAGS] = tags
            return self

        def chat_specials(self, specials):
            """Chat-markup markers that end a visible answer (a ChatSpecials or a list of strings)."""
            self._options[OPTION_CHAT_SPECIALS] = specials
            return self

        def listen(self, listener):
            """LlmListener for load progress (None: silent)."""
            self._options[OPTION_LISTENER] = listener
            return self

        def unpack_parameters(self, v: bool = True):
            """Expand packed weights to bf16 during this load (more device memory, the dense GEMM path); engines
            built on the model then never see packed tensors."""
            self._options[OPTION_UNPACK] = bool(v)
            return self

        def options(self, opts: dict):
            """Replace the load options map."""
            self._options = dict(opts or {})
            return self

        def device(self, d):
            self._device = d
            return self

        def build(self) -> LlmModel:
            if self._path is None:
                raise ValueError("path is required")
            return LlmModelFactory.make(self._path, self._options, self._device)

    @staticmethod
    def builder() -> "LlmModelFactory.Builder":
        return LlmModelFactory.Builder()

    @staticmethod
    def open(path) -> "LlmModelFactory.Builder":
        """``LlmModelFactory.open(path)...build()``: a builder bound to ``path``."""
        return LlmModelFactory.Builder().path(path)


# linear projections built by the layer classes (layers/linear.py), HF and GGUF tensor names
_PROJECTION = re.compile(r"(q_proj|k_proj|v_proj|o_proj|gate_proj|up_proj|down_proj|attn_q|attn_k|attn_v|"
                         r"attn_output|ffn_gate|ffn_up|ffn_down)\.weight$")


def _load_gguf(path: str, options, device, dtype) -> LlmModel:
    g = GgufFile(path)
    sel = MS.resolve_gguf(g.architecture)
    MS.check_source(sel, MS.SRC_GGUF, g.architecture, [])
    hf = hf_config_from_gguf(g.metadata, sel.architecture)
    tok = Tokenizer.from_gguf(g.metadata)
    weights: Dict[str, object] = {}
    packed = False
    # NVB_GGUF_PACKED=0 dequantizes every tensor at load time (the bf16 path); "force" keeps projections packed
    # on the CPU too (there they are dequantized per multiply -- for tests)
    mode = os.environ.get("NVB_GGUF_PACKED", "1")
    keep_packed = mode == "force" or (device.type == "cuda" and mode not in ("0", "false", "no"))
    if (options or {}).get(OPTION_UNPACK):
        keep_packed = False
    # under tensor parallelism the tensors stay in host memory until the model is built: each layer then moves
    # one tensor at a time to the GPU and keeps only its shard, so a rank's device memory peaks near its share
    # of the weights plus one full tensor (safetensors checkpoints are memory-mapped and behave the same way)
    from ..parallel import state as ps
    store = torch.device("cpu") if ps.tp_size() > 1 else device
    from ..utils.progress import LoadProgress
    prog = LoadProgress(f"GGUF {os.path.basename(path)}", len(g.tensors), (options or {}).get(OPTION_LISTENER))
    for name, info in g.tensors.items():
        prog.step(name)
        if sel.architecture == MS.QWEN3:
            target = hf_name_for_qwen3(name)
            if target is None:
                continue
        else:
            target = name
        packed = packed or info.ggml_type not in (0, 1, 30)
        if keep_packed and _PROJECTION.search(target) and fused_supported(info.ggml_type, info.shape):
            # projection weights stay in GGUF block format on the GPU (dequant-fused GEMM); the bytes are
            # copied out of the file mapping, which closes after loading
            raw = g.packed(name).to(store)
            weights[target] = GgufPacked(raw, info.ggml_type, info.shape[0], info.shape[1])
            continue
        weights[target] = g.get(name, dtype=torch.float32, device=store).to(dtype)
    if sel.architecture == MS.QWEN3 and "lm_head.weight" not in weights:
        hf.tie_word_embeddings = True
    g.close()
    prog.finish(f"{len(weights)} tensors")
    return LlmModel(hf, weights, tok, options, source=path, container="gguf", packed=packed)


def _load_hf_folder(d: str, options, device, dtype) -> LlmModel:
    cfg_path = os.path.join(d, "config.json")
    if not os.path.isfile(cfg_path):
        raise ModelLoadException(f"{d}: no config.json")
    hf = HfConfig.load(cfg_path)
    from ..loaders.onnx import normalize_bert_name, normalize_chat_name, read_initializers, select_file
    has_st = any(f.endswith(".safetensors") for f in os.listdir(d))
    onnx_file = None if has_st else select_file(d)
    source = MS.SRC_HF_SAFETENSORS if has_st else (MS.SRC_ONNX if onnx_file else None)
    if source is None:
        raise ModelLoadException(f"{d}: no *.safetensors or loadable *.onnx weights")
    sel = MS.require(hf, source)
    tok = Tokenizer.from_pretrained(d)
    if source == MS.SRC_HF_SAFETENSORS:
        if sel.architecture == MS.GEMMA4:
            from ..loaders.gemma4_qat import load_gemma4_qat
            weights = load_gemma4_qat(d, hf)
        else:
            from ..loaders.safetensors import SafetensorsCheckpoint
            from ..utils.progress import LoadProgress
            ck = SafetensorsCheckpoint(d)
            keys = ck.keys()
            prog = LoadProgress(f"safetensors {os.path.basename(d)}", len(keys), (options or {}).get(OPTION_LISTENER))
            weights = {}
            for k in keys:
                weights[k] = ck.get(k)
                prog.step(k)
            prog.finish(f"{len(keys)} tensors")
    else:
        raw = read_initializers(onnx_file)
        norm = normalize_bert_name if sel.architecture == MS.BERT else normalize_chat_name
        weights = {norm(k): v for k, v in raw.items()}
    if hf.tie_word_embeddings is False and "lm_head.weight" not in weights and sel.architecture != MS.BERT:
        hf.tie_word_embeddings = True
    return LlmModel(hf, weights, tok, options, source=d, container=source, packed=False)
