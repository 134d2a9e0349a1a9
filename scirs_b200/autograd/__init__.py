"""Graph-mode automatic differentiation with the reference's API
(scirs2-autograd: run / Context / placeholder / variable / grad /
Evaluator / Feeder / VariableEnvironment / tensor_ops / optimizers).

    from scirs_b200 import autograd as ag
    from scirs_b200.autograd import ops as T
"""
from . import ops, transforms  # noqa: F401
from .graph import Context, Evaluator, Feeder, Graph, Tensor, grad, run  # noqa: F401
from .transforms import (  # noqa: F401
    ExecutionTracer,
    GradientChecker,
    check_grad,
    hessian,
    hessian_vector_product,
    jacobian,
    jvp,
    scan,
    to_dot,
    to_json,
    to_mermaid,
    value_and_grad,
    vjp,
    vmap,
)
from .variables import SGD, AdaGrad, Adam, AdamW, MomentumSGD, VariableEnvironment  # noqa: F401
