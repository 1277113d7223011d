"""gRPC rotor twin (examples/rotor_twin_net): the ``rotor.RotorService``
service with ``SendFrame(Frame) -> Ack`` over grpcio, wire-compatible with
the reference's tonic/prost implementation (proto/rotor.proto)::

    message Frame { uint64 tick = 1; uint32 length = 2; float scale = 3; bytes residual = 4; }
    message Ack   { bool ok = 1; }

protoc is not available, so the two messages are encoded by hand (proto3
wire format: varints for tick/length/ok, fixed32 for scale, length-delimited
bytes; default values are omitted).  A negative ``scale`` marks a payload as
element RLE over INT16 codes (client.rs:86-108, server.rs:44-53).

Unlike the reference client, whose top-k path dequantizes the RLE bytes with
the plain error-bounded decoder and so drifts from the server (its closed
loop and the server's disagree), ``RotorClient`` updates its predictor with
exactly what the server reconstructs.
"""
from __future__ import annotations

import struct
import threading
import time
from concurrent import futures
from dataclasses import dataclass

import numpy as np

from ..ai.momentum import MomentumPredictor
from ..core.fixed_point import FixedPointBuffer
from ..hpc.quantizers import ErrorBoundedQuantizer, rle_decode_i16, rle_encode_i16

SERVICE = "rotor.RotorService"
METHOD = f"/{SERVICE}/SendFrame"


# ---------------------------------------------------------------- protobuf
def _varint(v: int) -> bytes:
    out = bytearray()
    v &= (1 << 64) - 1
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _read_varint(b: bytes, i: int) -> tuple[int, int]:
    v, shift = 0, 0
    while True:
        if i >= len(b):
            raise ValueError("truncated varint")
        c = b[i]
        i += 1
        v |= (c & 0x7F) << shift
        if not c & 0x80:
            return v, i
        shift += 7
        if shift > 63:
            raise ValueError("varint too long")


@dataclass
class Frame:
    tick: int = 0
    length: int = 0
    scale: float = 0.0
    residual: bytes = b""

    def encode(self) -> bytes:
        out = bytearray()
        if self.tick:
            out += b"\x08" + _varint(self.tick)
        if self.length:
            out += b"\x10" + _varint(self.length)
        if self.scale != 0.0:
            out += b"\x1d" + struct.pack("<f", self.scale)
        if self.residual:
            out += b"\x22" + _varint(len(self.residual)) + bytes(self.residual)
        return bytes(out)

    @classmethod
    def decode(cls, b: bytes) -> "Frame":
        f, i = cls(), 0
        while i < len(b):
            key, i = _read_varint(b, i)
            field, wt = key >> 3, key & 7
            if wt == 0:
                v, i = _read_varint(b, i)
                if field == 1:
                    f.tick = v
                elif field == 2:
                    f.length = v & 0xFFFFFFFF
            elif wt == 5:
                (v,) = struct.unpack_from("<f", b, i)
                i += 4
                if field == 3:
                    f.scale = v
            elif wt == 2:
                n, i = _read_varint(b, i)
                if field == 4:
                    f.residual = bytes(b[i:i + n])
                i += n
            elif wt == 1:
                i += 8
            else:
                raise ValueError(f"unsupported wire type {wt}")
        return f


def encode_ack(ok: bool) -> bytes:
    """Protobuf bytes of ``Ack { ok }`` (rotor.proto)."""
    return b"\x08\x01" if ok else b""


def decode_ack(b: bytes) -> bool:
    """Parse ``Ack`` bytes."""
    i, ok = 0, False
    while i < len(b):
        key, i = _read_varint(b, i)
        v, i = _read_varint(b, i)
        if key >> 3 == 1:
            ok = bool(v)
    return ok


def imu_sample(t: float) -> np.ndarray:
    """The client's synthetic 6-DOF IMU reading at time t (rotor_twin_net client.rs)."""
    w = np.float32(t) * np.float32(2.0) * np.float32(np.pi) * np.float32(1.67)
    s, c = np.sin(w), np.cos(w)
    return np.array([s, c, 0.01, s * np.float32(5.0), c * np.float32(5.0), 0.0], dtype=np.float32)


def _f32_display(x: np.float32) -> str:
    """An f32 as Rust's ``{}`` prints it: the shortest digits that read back
    as the same f32, positional, without a trailing ``.0`` (2.0 -> "2")."""
    return np.format_float_positional(np.float32(x), unique=True, trim="-")


# ------------------------------------------------------------------ server
class RotorServer:
    """Cloud side: predictor + error-bounded decoder; logs the reference's
    server CSV (``tick,..,len,..,raw,..,comp,..,ratio,..``)."""

    def __init__(self, beta: float = 0.9, epsilon: float = 0.05, metrics_path: str | None = None):
        self.pred = MomentumPredictor(beta)
        self.quant = ErrorBoundedQuantizer(epsilon)
        self.lock = threading.Lock()
        self.metrics = open(metrics_path, "w") if metrics_path else None
        self.last: np.ndarray | None = None
        self.frames = 0

    def handle(self, frame: Frame) -> bool:
        with self.lock:
            pred = self.pred.predict()
            if frame.scale < 0.0:
                codes = rle_decode_i16(frame.residual)
                deq = FixedPointBuffer.from_f32(codes.astype(np.float32) * np.float32(-frame.scale))
            else:
                deq = self.quant.dequantize(frame.residual, frame.scale)
            recon = deq if pred.is_empty() else pred.add(deq)
            vals = recon.to_f32()[: frame.length]
            rb = FixedPointBuffer.from_f32(vals)
            self.pred.update(rb)
            self.last = vals
            self.frames += 1
            if self.metrics:
                raw, comp = frame.length * 4, len(frame.residual) + 4
                ratio = float(np.float32(raw) / np.float32(comp))  # f32, as server.rs:70
                self.metrics.write(f"tick,{frame.tick},len,{frame.length},raw,{raw},comp,{comp},"
                                   f"ratio,{ratio:.4f}\n")
                self.metrics.flush()
        return True

    def serve(self, listen: str = "127.0.0.1:50051", max_workers: int = 4):
        import grpc

        server = grpc.server(futures.ThreadPoolExecutor(max_workers=max_workers))
        handler = grpc.method_handlers_generic_handler(SERVICE, {
            "SendFrame": grpc.unary_unary_rpc_method_handler(
                lambda req, ctx: self.handle(req), request_deserializer=Frame.decode,
                response_serializer=encode_ack),
        })
        server.add_generic_rpc_handlers((handler,))
        port = server.add_insecure_port(listen)
        server.start()
        return server, port


# ------------------------------------------------------------------ client
class RotorClient:
    """Edge side: predictor + error-bounded INT16 residuals (or top-k over
    the INT16 grid, RLE-packed, flagged by a negative scale)."""

    def __init__(self, target: str, epsilon: float = 0.05, topk: float = 0.0, beta: float = 0.9,
                 metrics_path: str | None = None):
        import grpc

        self.channel = grpc.insecure_channel(target)
        self.call = self.channel.unary_unary(METHOD, request_serializer=Frame.encode, response_deserializer=decode_ack)
        self.pred = MomentumPredictor(beta)
        self.quant = ErrorBoundedQuantizer(epsilon)
        self.epsilon = float(np.float32(epsilon))
        self.topk = topk
        self.metrics = open(metrics_path, "w") if metrics_path else None
        if self.metrics:
            self.metrics.write("tick,len,raw,comp,ratio\n")

    def encode(self, data: np.ndarray, tick: int) -> tuple[Frame, FixedPointBuffer]:
        buf = FixedPointBuffer.from_f32(data)
        pred = self.pred.predict()
        residual = buf.clone() if pred.is_empty() else buf.sub(pred)
        if self.topk > 0.0:
            res = residual.to_f32()
            n = res.size
            k = max(int(np.float32(n) * np.float32(self.topk)), 1)
            idx = np.argsort(-np.abs(res), kind="stable")[:k]
            scale = np.float32(2.0) * np.float32(self.epsilon)
            q = np.zeros(n, np.int16)
            # f32 quotient, rounded half away from zero (Rust's f32::round,
            # client.rs:99; numpy's round is half to even), clamped to i16
            d = (res[idx] / scale).astype(np.float64)
            q[idx] = np.clip(np.where(d < 0, -np.floor(0.5 - d), np.floor(d + 0.5)), -32768, 32767)
            payload, sc = rle_encode_i16(q), -float(scale)
            deq = FixedPointBuffer.from_f32(q.astype(np.float32) * scale)
        else:
            payload, sc = self.quant.quantize(residual)
            deq = self.quant.dequantize(payload, sc)
        recon = deq if pred.is_empty() else pred.add(deq)
        # Mirror the server exactly: it truncates to `length` through f32
        # before updating its predictor (server.rs:57-61).
        recon = FixedPointBuffer.from_f32(recon.to_f32()[: data.size])
        return Frame(tick, data.size, sc, payload), recon

    def send(self, data: np.ndarray, tick: int) -> bool:
        frame, recon = self.encode(data, tick)
        ok = self.call(frame, timeout=10.0)
        self.pred.update(recon)
        if self.metrics:
            raw, comp = data.size * 4, len(frame.residual) + 4
            self.metrics.write(f"{tick},{data.size},{raw},{comp},{_f32_display(np.float32(raw) / np.float32(comp))}\n")
        return ok

    def run(self, duration: float, rate_hz: int, sleep: bool = True) -> int:
        dt = 1.0 / max(rate_hz, 1)
        tick, t0 = 0, time.time()
        while True:
            t = (time.time() - t0) if sleep else tick * dt
            if t > duration:
                break
            self.send(imu_sample(t), tick)
            tick += 1
            if sleep:
                time.sleep(dt)
        return tick

    def close(self):
        self.channel.close()
        if self.metrics:
            self.metrics.close()
