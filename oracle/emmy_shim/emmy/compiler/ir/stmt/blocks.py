from emmy.compiler._model import Cond, Loop, StridedLoop  # noqa: F401
