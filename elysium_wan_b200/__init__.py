"""elysium_wan_b200: a Blackwell-native (sm_100a) pipeline-parallel GPT
training engine with the capabilities and public surface of wantrain
(virgiliolrf/elysium-wan)."""

__version__ = "0.1.0"
