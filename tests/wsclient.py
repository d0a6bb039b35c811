"""A minimal WebSocket client for the policy-server tests (RFC 6455 handshake and masked frames over a
plain socket) with openpi's msgpack_numpy packing: arrays travel as
{b"__ndarray__": True, b"data": bytes, b"dtype": str, b"shape": tuple}."""
import base64
import hashlib
import os
import socket
import struct

import msgpack
import numpy as np


def pack_array(obj):
    if isinstance(obj, np.ndarray):
        return {b"__ndarray__": True, b"data": obj.tobytes(), b"dtype": obj.dtype.str, b"shape": obj.shape}
    return obj


def unpack_array(obj):
    if b"__ndarray__" in obj:
        return np.ndarray(buffer=obj[b"data"], dtype=np.dtype(obj[b"dtype"]), shape=obj[b"shape"])
    return obj


def packb(x):
    return msgpack.packb(x, default=pack_array, use_bin_type=True)


def unpackb(b):
    return msgpack.unpackb(b, object_hook=unpack_array)


class Client:
    def __init__(self, port, host="127.0.0.1", timeout=300):
        self.s = socket.create_connection((host, port), timeout=timeout)
        key = base64.b64encode(os.urandom(16)).decode()
        self.s.sendall((f"GET / HTTP/1.1\r\nHost: {host}:{port}\r\nUpgrade: websocket\r\nConnection: Upgrade\r\n"
                        f"Sec-WebSocket-Key: {key}\r\nSec-WebSocket-Version: 13\r\n\r\n").encode())
        resp = b""
        while b"\r\n\r\n" not in resp:
            resp += self.s.recv(1)
        accept = base64.b64encode(hashlib.sha1((key + "258EAFA5-E914-47DA-95CA-C5AB0DC85B11").encode()).digest())
        assert resp.startswith(b"HTTP/1.1 101") and accept in resp, resp
        self.metadata = unpackb(self.recv())

    def _read(self, n):
        buf = b""
        while len(buf) < n:
            chunk = self.s.recv(n - len(buf))
            if not chunk:
                raise ConnectionError("closed")
            buf += chunk
        return buf

    def send(self, payload, opcode=0x2, fragment=None):
        """one message, optionally split into frames of `fragment` bytes (continuation frames)"""
        parts = [payload] if not fragment else [payload[i:i + fragment] for i in range(0, len(payload), fragment)]
        for i, part in enumerate(parts):
            op = opcode if i == 0 else 0x0
            fin = 0x80 if i == len(parts) - 1 else 0
            mask = os.urandom(4)
            n = len(part)
            hdr = bytes([fin | op])
            if n < 126:
                hdr += bytes([0x80 | n])
            elif n < 65536:
                hdr += bytes([0x80 | 126]) + struct.pack(">H", n)
            else:
                hdr += bytes([0x80 | 127]) + struct.pack(">Q", n)
            body = bytes(b ^ mask[j & 3] for j, b in enumerate(part)) if n < 4096 else \
                (np.frombuffer(part, np.uint8) ^ np.resize(np.frombuffer(mask, np.uint8), n)).tobytes()
            self.s.sendall(hdr + mask + body)

    def recv(self):
        h = self._read(2)
        n = h[1] & 0x7F
        if n == 126:
            n = struct.unpack(">H", self._read(2))[0]
        elif n == 127:
            n = struct.unpack(">Q", self._read(8))[0]
        return self._read(n)

    def call(self, obj, fragment=None):
        self.send(packb(obj), fragment=fragment)
        return unpackb(self.recv())

    def close(self):
        try:
            self.send(b"", opcode=0x8)
        finally:
            self.s.close()


def http_get(port, path, host="127.0.0.1"):
    with socket.create_connection((host, port), timeout=60) as s:
        s.sendall(f"GET {path} HTTP/1.1\r\nHost: {host}\r\n\r\n".encode())
        out = b""
        while True:
            chunk = s.recv(4096)
            if not chunk:
                return out
            out += chunk
