"""A backend for the reference's ``InferenceSession`` that runs on this library.

The reference's sessions drive a ``Backend`` (src/aexrt/backends/base.py:21-37): ``info()``,
``prepare(graph)`` and ``run(inputs) -> outputs``, chosen by ``InferenceSession._make_backend``
(src/aexrt/session.py:33-51).  ``B200Backend`` has the same three methods:

* ``prepare`` takes an ``.aexrt`` path, engine bytes, or a reference ``Graph``; a graph is compiled
  by the reference's own ``build_aexrt_engine`` (the compile surface stays the reference's: pass
  ``algo_overrides={command: 51|52|53}`` and ``int8_pergroup=[...]`` to select the W8A8 kernels),
  then the engine is loaded through the runtime ABI (aexrt_yolo_load_engine);
* ``run`` takes ``{input name: NCHW images}`` (fp32 or fp16, any batch the model was prepared for)
  and returns ``{output name: output0}``; the detections of the run are kept on
  ``last_detections`` as (rows [images, max_detections, 6], counts [images]).
"""
from __future__ import annotations

import os
import tempfile
from dataclasses import dataclass, field
from typing import Any, Dict, Optional

import numpy as np


@dataclass(frozen=True)
class BackendInfo:
    """The fields of the reference's BackendInfo (src/aexrt/backends/base.py:11-18)."""

    name: str
    device: str
    capabilities: Dict[str, Any] = field(default_factory=dict)


class B200Backend:
    name = "b200"
    supported_ops = frozenset({"Conv", "Sigmoid", "Mul", "Add", "Concat", "Split", "Resize", "MaxPool", "Reshape",
                               "Transpose", "Softmax", "Slice", "Sub", "Div"})
    supported_dtypes = frozenset({"float32", "float16"})
    supported_features = frozenset({"w8a8", "cuda_graph", "yolo_postprocess"})

    def __init__(self, device_index: int = 0, images: Optional[int] = None, **compile_kwargs):
        self.device_index = device_index
        self.images = images
        self.compile_kwargs = compile_kwargs
        self.model = None
        self.input_name = "images"
        self.output_name = "output0"
        self.last_detections = None

    def info(self) -> BackendInfo:
        caps = {"sm": "100a", "int8_tensor_cores": True, "max_detections": 100}
        if self.model is not None:
            caps.update(self.model.capabilities)
        return BackendInfo(self.name, f"cuda:{self.device_index}", caps)

    @staticmethod
    def compile(graph, **kwargs) -> bytes:
        """Engine bytes of a reference Graph, compiled by the reference's build_aexrt_engine (the
        reference package must be importable) and validated by this library's loader."""
        import aexrt  # the reference package

        from .cpp_runtime import validate_engine

        data = aexrt.build_aexrt_engine(graph, **kwargs)
        validate_engine(data)
        return data

    def prepare(self, graph) -> None:
        from .cpp_runtime import NativeCppYoloModel

        if isinstance(graph, (str, os.PathLike)):
            path = os.fspath(graph)
        else:
            data = bytes(graph) if isinstance(graph, (bytes, bytearray)) else self.compile(graph, **self.compile_kwargs)
            if not isinstance(graph, (bytes, bytearray)):
                self.input_name = next(iter(graph.inputs))
                self.output_name = graph.outputs[0]
            fd, path = tempfile.mkstemp(suffix=".aexrt")
            with os.fdopen(fd, "wb") as f:
                f.write(data)
        self.model = NativeCppYoloModel(path, self.device_index, images=self.images)

    def run(self, inputs: Dict[str, Any]) -> Dict[str, Any]:
        if self.model is None:
            raise RuntimeError("prepare() the backend first")
        x = inputs[self.input_name] if self.input_name in inputs else next(iter(inputs.values()))
        x = np.asarray(x)
        rows, counts = self.model.run_batch(x if x.dtype == np.float16 else x.astype(np.float32))
        self.last_detections = (rows, counts)
        return {self.output_name: self.model.output0()}

    def close(self) -> None:
        if self.model is not None:
            self.model.close()
            self.model = None
