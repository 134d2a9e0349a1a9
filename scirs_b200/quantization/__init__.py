"""Quantization: int8 / int4 formats, GPTQ, AWQ, SmoothQuant, calibration
observers, post-training quantization and quantization-aware training."""
from .core import (GroupSize, Granularity, Int4Tensor, Int8Mode, Int8Tensor, QuantizationConfig, QuantizationMode,
                   QuantizationParams, QuantizationScheme, QuantizedTensor, dequantize_int4, dequantize_int8,
                   fake_quantize, int4_roundtrip_mse, quantize_int4, quantize_int8, quantized_matmul, roundtrip_mse)
from .methods import (ActivationStats, AwqConfig, AwqQuantizedLayer, AwqQuantizer, CalibrationRunner,
                      FakeQuantLinear, GptqConfig, GptqQuantizer, GptqResult, MinMaxObserver, MovingAverageObserver,
                      ObserverStats, PercentileObserver, PostTrainingQuantizer, QuantizationAwareTraining,
                      SmoothQuantConfig, minmax_calibration_runner, naive_quantize, smooth_linear, smooth_scales)
