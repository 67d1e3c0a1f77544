"""Pick the network interface that reaches the rendezvous host (reference ``utils/network.py:8-34``)."""

from __future__ import annotations

import socket


def interface_addresses():
    """{interface name: IPv4 address} from the host's interfaces (Linux)."""
    import fcntl
    import struct
    out = {}
    for _, name in socket.if_nameindex():
        s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
        try:
            packed = fcntl.ioctl(s.fileno(), 0x8915, struct.pack("256s", name[:15].encode()))  # SIOCGIFADDR
            out[name] = socket.inet_ntoa(packed[20:24])
        except OSError:
            pass
        finally:
            s.close()
    return out


def rendezvous_interface(master):
    """Interface whose address routes to ``master`` (the source address the kernel picks)."""
    addresses = interface_addresses()
    s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
    try:
        s.connect((socket.gethostbyname(master), 9))
        local = s.getsockname()[0]
    finally:
        s.close()
    for name, addr in addresses.items():
        if addr == local:
            return name, addresses
    raise RuntimeError(f"no interface routes to {master} (source address {local})")
