"""backends"""
