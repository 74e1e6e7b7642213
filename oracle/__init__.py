# SPDX-License-Identifier: Apache-2.0
"""Test-infrastructure oracle for kotflash_b200 (never imported by the product)."""
