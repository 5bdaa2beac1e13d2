"""Typed exception hierarchy of the library.

Mirrors the reference's exception tree (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/exceptions/*.java):
``NanoLlvmException`` is the root, ``ModelLoadException`` covers every load failure and
``UnsupportedModelException`` narrows it to architecture / container rejections.  Generation ends with
``GenerationCancelledException`` after ``LLM.cancel()`` and with ``GenerationTimeoutException`` when the
wall-clock deadline passes; both are raised between engine steps, never from inside a kernel.

``DeviceWaitTimeout`` is new: fused multi-GPU kernels wait on peer flags with a bounded spin and report a
timeout through an error word that the host turns into this exception.  ``TensorParallelAbort`` is new too:
a tensor-parallel rank whose step failed publishes the reason and every other rank raises this between steps.
"""


class NanoLlvmException(RuntimeError):
    """Root of all library errors."""


class ModelLoadException(NanoLlvmException):
    """A checkpoint could not be read, bound or filled."""


class UnsupportedModelException(ModelLoadException):
    """The checkpoint is readable but its architecture or container combination is rejected."""


class GenerationCancelledException(NanoLlvmException):
    """``LLM.cancel()`` was called while a generate call was running."""


class GenerationTimeoutException(NanoLlvmException):
    """The generate call exceeded its wall-clock deadline."""


class DeviceWaitTimeout(NanoLlvmException):
    """A device-side bounded wait (peer flag, mbarrier) gave up; the kernel returned an error status."""


class TensorParallelAbort(NanoLlvmException):
    """Another tensor-parallel rank failed; this rank stops before launching its next step."""


class StepInputError(NanoLlvmException):
    """Debug-mode step check: an index the kernels would use as an address is out of range, or two sequences of
    one step would write the same KV page (a data race) -- caught on the host before any kernel runs."""
