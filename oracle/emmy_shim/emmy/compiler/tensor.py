from emmy.compiler._model import Tensor  # noqa: F401
