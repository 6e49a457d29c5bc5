"""TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's pn_fir_tau
algorithm, used by tests/, __graft_entry__.smoke() and bench.py's CPU legs as
the checker or the timed CPU baseline. Never imported by the product package.
"""
