from emmy.compiler._model import BinaryExpr, Expr, FlatIndex, Literal, TernaryExpr, Var  # noqa: F401
