"""Plans, workspaces, packed weights and the dispatch gate (B200 runtime).

Drop-in for ``src/rdna3_fastmm/runtime.py`` of chelokot/rdna3-fastmm
(``Rank7Plan``, ``Rank48Plan``, ``Rank49Plan``, ``Workspace``,
``PackedWeight``, ``LinearShapeFamily``, ``unsupported_runtime_reason``,
``is_tested_runtime``): same constructor arguments, methods, properties,
validation order and error types (``ValueError`` for arguments,
``MemoryError`` for the free-memory budget).  Execution goes through
``libfmm_sm100.so``; nothing here computes on the CPU.

B200-specific differences, all deliberate:

* transformed weight planes are stored K-major, ``[rank, bn, ldk]`` (the
  transpose of the reference's ``[rank, bk, bn]``), which is the operand layout
  of the tcgen05 leaf GEMM;
* plane rows are padded to a multiple of 8 elements (``ldk``, ``ldp``) so every
  TMA row starts on a 16-byte boundary; byte counts include that padding and
  equal the reference's formulas whenever ``bk`` and ``bn`` are multiples of 8;
* the dispatch tables hold shapes measured on B200 against cuBLAS BF16.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native
from .schemes import get_scheme

__all__ = [
    "MatrixShape",
    "Workspace",
    "PackedWeight",
    "PackedRight",
    "LinearShapeFamily",
    "ElementTransformConfig",
    "WeightTransformConfig",
    "Rank7Plan",
    "Rank343Plan",
    "Rank48Plan",
    "Rank49Plan",
    "Rank7Workspace",
    "Rank49Workspace",
    "unsupported_runtime_reason",
    "is_tested_runtime",
]


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def _round_up(a: int, b: int) -> int:
    return _cdiv(a, b) * b


@dataclass(frozen=True)
class MatrixShape:
    """Block dimensions of an ``M x K x N`` product for an ``s x s`` scheme.

    Mirrors ``MatrixShape`` (reference ``runtime.py:56-89``) and adds the
    16-byte row pitches of the FP16 planes.
    """

    rows: int
    inner: int
    columns: int
    block_rows: int
    block_inner: int
    block_columns: int

    @classmethod
    def from_dimensions(cls, rows: int, inner: int, columns: int, scheme_size: int) -> "MatrixShape":
        if min(rows, inner, columns) < 1:
            raise ValueError("matrix dimensions must be positive")
        return cls(rows, inner, columns, _cdiv(rows, scheme_size), _cdiv(inner, scheme_size),
                   _cdiv(columns, scheme_size))

    @property
    def dimensions(self) -> tuple[int, int, int]:
        return self.rows, self.inner, self.columns

    @property
    def inner_pitch(self) -> int:
        """Row pitch (elements) of the left and right planes."""
        return _round_up(self.block_inner, 8)

    @property
    def column_pitch(self) -> int:
        """Row pitch (elements) of the product planes."""
        return _round_up(self.block_columns, 8)

    def workspace_elements(self, rank: int) -> int:
        """Logical elements of L, R and P (reference formula, no padding)."""
        return rank * (
            self.block_rows * self.block_inner
            + self.block_inner * self.block_columns
            + self.block_rows * self.block_columns
        )


@dataclass
class Workspace:
    algorithm: str
    output_dtype: torch.dtype
    compute_dtype: torch.dtype
    left_transformed: torch.Tensor  # [rank, bm, ldk]
    right_transformed: torch.Tensor | None  # [rank, bn, ldk] (K-major)
    products: torch.Tensor  # [rank, bm, ldp]


@dataclass(frozen=True)
class _PackedTransform:
    algorithm: str
    source_dtype: torch.dtype
    compute_dtype: torch.dtype
    transformed: torch.Tensor  # [rank, bn, ldk]
    source_shape: tuple[int, int]


@dataclass(frozen=True)
class PackedRight(_PackedTransform):
    pass


@dataclass(frozen=True)
class PackedWeight(_PackedTransform):
    pass


@dataclass(frozen=True)
class LinearShapeFamily:
    minimum_rows: int
    maximum_rows: int
    inner: int
    columns: int
    has_bias: bool

    def matches(self, shape: tuple[int, int, int], has_bias: bool) -> bool:
        rows, inner, columns = shape
        return (
            self.minimum_rows <= rows <= self.maximum_rows
            and inner == self.inner
            and columns == self.columns
            and has_bias == self.has_bias
        )


@dataclass(frozen=True)
class ElementTransformConfig:
    """Launch geometry of a streaming transform: elements per thread-vector
    and threads per block (the B200 counterpart of the reference's
    block_elements/warps pair)."""

    vector_elements: int
    threads: int


@dataclass(frozen=True)
class WeightTransformConfig:
    vector_elements: int
    threads: int


class _LinearPlan:
    algorithm: str
    scheme: str
    rank: int
    scheme_size: int
    precision_pairs: frozenset
    # plain-mm API tables (FP16 in, FP16 out): shapes measured to win on B200
    dynamic_shapes: frozenset = frozenset()
    prepacked_shapes: frozenset = frozenset()
    linear_shape_families: tuple[LinearShapeFamily, ...] = ()
    prepacked_linear_shape_families: tuple[LinearShapeFamily, ...] = ()
    transform_vector: int = 4

    def __init__(
        self,
        rows: int,
        inner: int,
        columns: int,
        device: torch.device,
        dtype: torch.dtype = torch.float16,
        compute_dtype: torch.dtype | None = None,
    ) -> None:
        device = torch.device(device)
        if device.type != "cuda" or torch.version.cuda is None or not torch.cuda.is_available():
            raise ValueError("the B200 backend requires a CUDA sm_100 device")
        resolved = dtype if compute_dtype is None else compute_dtype
        if (dtype, resolved) not in self.precision_pairs:
            raise ValueError(
                f"{self.algorithm} does not support {dtype} inputs with {resolved} leaf products"
            )
        index = torch.cuda.current_device() if device.index is None else device.index
        self.device = torch.device("cuda", index)
        self.dtype = dtype
        self.compute_dtype = resolved
        self.shape = MatrixShape.from_dimensions(rows, inner, columns, self.scheme_size)

    # ------------------------------------------------------------------ sizes
    @property
    def workspace_bytes(self) -> int:
        return self._workspace_bytes(prepacked_right=False)

    @property
    def prepacked_workspace_bytes(self) -> int:
        return self._workspace_bytes(prepacked_right=True)

    @property
    def packed_right_bytes(self) -> int:
        s = self.shape
        return self.rank * s.block_columns * s.inner_pitch * self.compute_dtype.itemsize

    @property
    def packed_weight_bytes(self) -> int:
        return self.packed_right_bytes

    def _workspace_bytes(self, prepacked_right: bool) -> int:
        s = self.shape
        elements = self.rank * (s.block_rows * s.inner_pitch + s.block_rows * s.column_pitch)
        if not prepacked_right:
            elements += self.rank * s.block_columns * s.inner_pitch
        return elements * self.compute_dtype.itemsize

    # ------------------------------------------------------------------ gate
    def is_recommended(self, *, prepacked_right: bool = False) -> bool:
        """Plain-mm gate (reference ``runtime.py:207-214``)."""
        shapes = self.prepacked_shapes if prepacked_right else self.dynamic_shapes
        return (
            self.dtype == torch.float16
            and self.compute_dtype == torch.float16
            and self.shape.dimensions in shapes
            and is_tested_runtime(self.device)
        )

    @classmethod
    def has_measured_linear_win(cls, shape: tuple[int, int, int], *, has_bias: bool,
                                prepacked_weight: bool = False) -> bool:
        families = cls.linear_shape_families
        if prepacked_weight:
            families = families + cls.prepacked_linear_shape_families
        return any(family.matches(shape, has_bias) for family in families)

    def is_linear_recommended(self, *, has_bias: bool, prepacked_weight: bool = False) -> bool:
        return (
            self.dtype == torch.bfloat16
            and self.compute_dtype == torch.float16
            and self.has_measured_linear_win(self.shape.dimensions, has_bias=has_bias,
                                             prepacked_weight=prepacked_weight)
            and is_tested_runtime(self.device)
        )

    @classmethod
    def transform_config(cls, inner: int, columns: int) -> ElementTransformConfig:
        return ElementTransformConfig(cls.transform_vector, 256)

    @classmethod
    def weight_transform_config(cls, inner: int, columns: int) -> WeightTransformConfig:
        return WeightTransformConfig(cls.transform_vector, 256)

    # ------------------------------------------------------------------ memory
    def _ensure_memory_budget(self, required: int, fraction: float, name: str) -> None:
        if not 0 < fraction <= 1:
            raise ValueError("memory fraction must be in the interval (0, 1]")
        free, _ = torch.cuda.mem_get_info(self.device)
        budget = free * fraction
        if required > budget:
            raise MemoryError(
                f"{name} needs {required / 2**30:.2f} GiB, exceeding the {budget / 2**30:.2f} GiB budget"
            )

    def _planes(self, kind: str) -> torch.Tensor:
        s = self.shape
        shape = {
            "left": (self.rank, s.block_rows, s.inner_pitch),
            "right": (self.rank, s.block_columns, s.inner_pitch),
            "products": (self.rank, s.block_rows, s.column_pitch),
        }[kind]
        return torch.empty(shape, device=self.device, dtype=self.compute_dtype)

    def allocate_workspace(self, max_free_memory_fraction: float = 0.75, *,
                           prepacked_right: bool = False) -> Workspace:
        self._ensure_memory_budget(self._workspace_bytes(prepacked_right), max_free_memory_fraction,
                                   f"{self.algorithm} workspace")
        return Workspace(
            algorithm=self.algorithm,
            output_dtype=self.dtype,
            compute_dtype=self.compute_dtype,
            left_transformed=self._planes("left"),
            right_transformed=None if prepacked_right else self._planes("right"),
            products=self._planes("products"),
        )

    def pack_weight(self, weight: torch.Tensor, max_free_memory_fraction: float = 0.75) -> PackedWeight:
        """Transform the weight once on the device into an immutable snapshot."""
        self._validate_weight(weight)
        self._ensure_memory_budget(self.packed_weight_bytes, max_free_memory_fraction,
                                   f"{self.algorithm} packed Linear weight")
        transformed = self._planes("right")
        with torch.cuda.device(self.device):
            _native.transform_w(self.scheme, weight, transformed)
        s = self.shape
        return PackedWeight(self.algorithm, self.dtype, self.compute_dtype, transformed,
                            (s.columns, s.inner))

    def pack_right(self, right: torch.Tensor, max_free_memory_fraction: float = 0.75) -> PackedRight:
        """Transform a contiguous right matrix ``[K, N]`` once on the device."""
        self._validate_right(right)
        self._ensure_memory_budget(self.packed_right_bytes, max_free_memory_fraction,
                                   f"{self.algorithm} packed right matrix")
        transformed = self._planes("right")
        with torch.cuda.device(self.device):
            _native.transform_b(self.scheme, right, transformed)
        s = self.shape
        return PackedRight(self.algorithm, self.dtype, self.compute_dtype, transformed, (s.inner, s.columns))

    # ------------------------------------------------------------------ run
    def run(self, left: torch.Tensor, right: torch.Tensor, workspace: Workspace,
            output: torch.Tensor | None = None) -> torch.Tensor:
        """``left @ right`` for contiguous ``left[M, K]`` and ``right[K, N]``
        (reference ``runtime.py:278-308``)."""
        self._validate_left(left)
        self._validate_right(right)
        self._validate_workspace(workspace, require_right=True)
        result = self._output(output)
        self._validate_output_storage(result, left, right, workspace.left_transformed,
                                      workspace.products, workspace.right_transformed)
        right_planes = workspace.right_transformed
        if right_planes is None:
            raise ValueError("dynamic execution requires a dynamic workspace")
        with torch.cuda.device(self.device):
            _native.linear(self.scheme, left, right, None, result, workspace.left_transformed,
                           right_planes, workspace.products, prepacked=False, right_kn=True)
        return result

    def run_packed(self, left: torch.Tensor, right: PackedRight, workspace: Workspace,
                   output: torch.Tensor | None = None) -> torch.Tensor:
        """``left @ right`` with the right matrix packed by ``pack_right``
        (reference ``runtime.py:310-341``)."""
        self._validate_left(left)
        self._validate_packed_right(right)
        self._validate_workspace(workspace, require_right=False)
        result = self._output(output)
        self._validate_separate_storage(right.transformed, workspace.left_transformed, workspace.products)
        self._validate_output_storage(result, left, right.transformed, workspace.left_transformed,
                                      workspace.products, workspace.right_transformed)
        with torch.cuda.device(self.device):
            _native.linear(self.scheme, left, None, None, result, workspace.left_transformed,
                           right.transformed, workspace.products, prepacked=True)
        return result

    def run_linear(self, input_tensor: torch.Tensor, weight: torch.Tensor, workspace: Workspace,
                   bias: torch.Tensor | None = None, output: torch.Tensor | None = None) -> torch.Tensor:
        self._validate_left(input_tensor)
        self._validate_weight(weight)
        if bias is not None:
            self._validate_bias(bias)
        self._validate_workspace(workspace, require_right=True)
        result = self._output(output)
        self._validate_output_storage(result, input_tensor, weight, bias, workspace.left_transformed,
                                      workspace.products, workspace.right_transformed)
        right = workspace.right_transformed
        if right is None:
            raise ValueError("linear execution requires a dynamic workspace")
        with torch.cuda.device(self.device):
            _native.linear(self.scheme, input_tensor, weight, bias, result,
                           workspace.left_transformed, right, workspace.products, prepacked=False)
        return result

    def run_linear_packed(self, input_tensor: torch.Tensor, weight: PackedWeight, workspace: Workspace,
                          bias: torch.Tensor | None = None,
                          output: torch.Tensor | None = None) -> torch.Tensor:
        self._validate_left(input_tensor)
        self._validate_packed_weight(weight)
        if bias is not None:
            self._validate_bias(bias)
        self._validate_workspace(workspace, require_right=False)
        self._validate_separate_storage(weight.transformed, workspace.left_transformed,
                                        workspace.products)
        result = self._output(output)
        self._validate_output_storage(result, input_tensor, weight.transformed, bias,
                                      workspace.left_transformed, workspace.products,
                                      workspace.right_transformed)
        with torch.cuda.device(self.device):
            _native.linear(self.scheme, input_tensor, None, bias, result, workspace.left_transformed,
                           weight.transformed, workspace.products, prepacked=True)
        return result

    # ------------------------------------------------------------------ checks
    def _validate_left(self, tensor: torch.Tensor) -> None:
        self._validate_tensor(tensor, (self.shape.rows, self.shape.inner), "left")

    def _validate_right(self, tensor: torch.Tensor) -> None:
        self._validate_tensor(tensor, (self.shape.inner, self.shape.columns), "right")

    def _validate_weight(self, tensor: torch.Tensor) -> None:
        self._validate_tensor(tensor, (self.shape.columns, self.shape.inner), "weight")

    def _validate_bias(self, tensor: torch.Tensor) -> None:
        self._validate_tensor(tensor, (self.shape.columns,), "bias")

    def _validate_tensor(self, tensor: torch.Tensor, shape: tuple[int, ...], name: str) -> None:
        if tuple(tensor.shape) != shape:
            raise ValueError(f"{name} matrix has shape {tuple(tensor.shape)}, expected {shape}")
        if tensor.device != self.device or tensor.dtype != self.dtype:
            raise ValueError(f"{name} matrix device or dtype does not match the plan")
        if not tensor.is_contiguous():
            raise ValueError(f"{name} matrix must be contiguous")
        if tensor.requires_grad:
            raise ValueError("the B200 fast-matmul backend does not support autograd")

    def _validate_workspace(self, workspace: Workspace, *, require_right: bool) -> None:
        if (workspace.algorithm != self.algorithm or workspace.output_dtype != self.dtype
                or workspace.compute_dtype != self.compute_dtype):
            raise ValueError("workspace does not match the plan")
        s = self.shape
        expected = [
            (workspace.left_transformed, (self.rank, s.block_rows, s.inner_pitch)),
            (workspace.products, (self.rank, s.block_rows, s.column_pitch)),
        ]
        if require_right:
            if workspace.right_transformed is None:
                raise ValueError("dynamic execution requires a dynamic workspace")
            expected.append((workspace.right_transformed, (self.rank, s.block_columns, s.inner_pitch)))
        for tensor, shape in expected:
            if (tuple(tensor.shape) != shape or tensor.device != self.device
                    or tensor.dtype != self.compute_dtype or not tensor.is_contiguous()
                    or tensor.requires_grad):
                raise ValueError("workspace does not match the plan")
        self._validate_separate_storage(*(tensor for tensor, _ in expected))

    def _validate_packed_weight(self, packed: PackedWeight) -> None:
        if not isinstance(packed, PackedWeight):
            raise ValueError("packed Linear weight does not match the plan")
        s = self.shape
        self._validate_packed(packed, (s.columns, s.inner), "Linear weight")

    def _validate_packed_right(self, packed: PackedRight) -> None:
        if not isinstance(packed, PackedRight):
            raise ValueError("packed right matrix does not match the plan")
        s = self.shape
        self._validate_packed(packed, (s.inner, s.columns), "right matrix")

    def _validate_packed(self, packed: _PackedTransform, source_shape: tuple[int, int], name: str) -> None:
        if (packed.algorithm != self.algorithm or packed.source_dtype != self.dtype
                or packed.compute_dtype != self.compute_dtype):
            raise ValueError(f"packed {name} does not match the plan")
        s = self.shape
        if packed.source_shape != source_shape:
            raise ValueError(f"packed {name} shape does not match the plan")
        t = packed.transformed
        if (tuple(t.shape) != (self.rank, s.block_columns, s.inner_pitch) or t.device != self.device
                or t.dtype != self.compute_dtype or not t.is_contiguous() or t.requires_grad):
            raise ValueError(f"packed {name} does not match the plan")

    def _output(self, output: torch.Tensor | None) -> torch.Tensor:
        shape = (self.shape.rows, self.shape.columns)
        if output is None:
            return torch.empty(shape, device=self.device, dtype=self.dtype)
        self._validate_tensor(output, shape, "output")
        return output

    def _validate_output_storage(self, output: torch.Tensor, *tensors: torch.Tensor | None) -> None:
        for tensor in tensors:
            if tensor is not None and _overlaps(output, tensor):
                raise ValueError("output storage must not overlap inputs or workspace")

    def _validate_separate_storage(self, *tensors: torch.Tensor) -> None:
        for i, tensor in enumerate(tensors):
            if any(_overlaps(tensor, other) for other in tensors[i + 1:]):
                raise ValueError("work buffers must not overlap")


def _overlaps(first: torch.Tensor, second: torch.Tensor) -> bool:
    a0 = first.data_ptr()
    a1 = a0 + first.numel() * first.element_size()
    b0 = second.data_ptr()
    b1 = b0 + second.numel() * second.element_size()
    return a0 < b1 and b0 < a1


_BF16_FP16 = frozenset({(torch.bfloat16, torch.float16)})
# FP16 inputs with FP16 leaves, as the reference's rank-7 and rank-49 plans
# allow; BF16 leaf products (the reference's (bf16, bf16) rank-49 pair) are not
# built for B200
_FP16_AND_BF16_FP16 = frozenset({(torch.float16, torch.float16), (torch.bfloat16, torch.float16)})


class Rank7Plan(_LinearPlan):
    """``<2,2,2>`` rank-7 scheme (reference ``runtime.py:780-820``)."""

    algorithm = "rank7-v1"
    scheme = "rank7"
    rank = 7
    scheme_size = 2
    precision_pairs = _FP16_AND_BF16_FP16
    transform_vector = 8
    # B200 measurements against cuBLAS BF16 (F.linear): no shape has won yet,
    # so nothing is routed here by the graph rewrite.
    linear_shape_families: tuple[LinearShapeFamily, ...] = ()
    prepacked_linear_shape_families: tuple[LinearShapeFamily, ...] = ()


class Rank48Plan(_LinearPlan):
    """``<4,4,4>`` rank-48 dyadic SLP scheme (reference ``runtime.py:823-844``)."""

    algorithm = "rank48-accurate-v1"
    scheme = "rank48"
    rank = 48
    scheme_size = 4
    precision_pairs = _BF16_FP16
    linear_shape_families: tuple[LinearShapeFamily, ...] = ()
    prepacked_linear_shape_families: tuple[LinearShapeFamily, ...] = ()


class Rank49Plan(_LinearPlan):
    """``<4,4,4>`` rank-49 scheme (reference ``runtime.py:847-880``)."""

    algorithm = "rank49-v1"
    scheme = "rank49"
    rank = 49
    scheme_size = 4
    # (bfloat16, bfloat16): BF16 planes, BF16 leaf products (tcgen05 with BF16
    # operands), as the reference's pair of the same name
    precision_pairs = _FP16_AND_BF16_FP16 | frozenset({(torch.bfloat16, torch.bfloat16)})
    linear_shape_families: tuple[LinearShapeFamily, ...] = ()
    prepacked_linear_shape_families: tuple[LinearShapeFamily, ...] = ()


class Rank343Plan(_LinearPlan):
    """``<8,8,8>`` rank-343 scheme for FP16 square products
    (reference ``runtime.py:883-962``): FP16 inputs and output only, the
    plain-mm API (``run``, ``pack_right``, ``run_packed``).  The output side is
    the +-1 coefficient sum over the 343 products (the reference uses a matrix
    product against the same coefficients).  No shape is admitted by
    ``is_recommended`` until one measures faster than cuBLAS FP16 on B200."""

    algorithm = "rank343-mfma-v1"
    scheme = "rank343"
    rank = 343
    scheme_size = 8
    precision_pairs = frozenset({(torch.float16, torch.float16)})
    transform_vector = 2
    dynamic_shapes: frozenset = frozenset()
    prepacked_shapes: frozenset = frozenset()


for _plan in (Rank7Plan, Rank48Plan, Rank49Plan, Rank343Plan):
    _scheme = get_scheme(_plan.scheme)
    assert (_scheme.rank, _scheme.size) == (_plan.rank, _plan.scheme_size), _plan

Rank7Workspace = Workspace
Rank49Workspace = Workspace

TESTED_TORCH_PREFIX = "2.11."
TESTED_CUDA_PREFIX = "12."


def unsupported_runtime_reason(device: torch.device | None = None) -> str | None:
    """Why this runtime is not the one the dispatch tables were measured on
    (``None`` when it is).  Mirrors the reference's pin
    (``runtime.py:970-994``) for sm_100 / 148 SMs / torch 2.11 / CUDA 12."""
    if torch.version.cuda is None:
        return "requires a CUDA PyTorch build"
    if not torch.cuda.is_available():
        return "requires an available CUDA GPU"
    resolved = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if resolved.type != "cuda":
        return "requires a CUDA GPU device"
    props = torch.cuda.get_device_properties(resolved)
    capability = (props.major, props.minor)
    if capability != (10, 0) or props.multi_processor_count != 148:
        return (
            "tested only on sm_100 with 148 SMs; found "
            f"sm_{props.major}{props.minor} with {props.multi_processor_count}"
        )
    if not torch.__version__.startswith(TESTED_TORCH_PREFIX):
        return f"tested only with PyTorch 2.11; found {torch.__version__}"
    if not str(torch.version.cuda).startswith(TESTED_CUDA_PREFIX):
        return f"tested only with CUDA 12; found {torch.version.cuda}"
    try:
        _native.library()
    except _native.NativeLibraryError as error:
        return str(error)
    return None


def is_tested_runtime(device: torch.device) -> bool:
    return unsupported_runtime_reason(device) is None
