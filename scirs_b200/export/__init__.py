"""Model export: ONNX (protobuf and JSON) and raw weight files."""
from .onnx import (OnnxGraph, OnnxModel, OnnxNode, OnnxTensor, OnnxValueInfo, export_activation, export_batchnorm,
                   export_conv2d, export_linear, export_sequential, run_graph)
