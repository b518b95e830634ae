"""B200-native XINT8 YOLOv8 and W4A8 inference engine (sm_100a)."""
from .graph import ConvLayer, GraphIR, PoolLayer, Segment, SigmoidFit, TensorInfo  # noqa: F401
from .yolov8 import HEAD_NAMES, ModelSpec, build_yolov8, random_images  # noqa: F401
from .session import GraphSession, InferenceSession, RunHandle, save_graph  # noqa: F401
