#:set architecture = [('Transpose', ['input'], [[2, 1, 3]]), ('LSTM', ['input', 'hidden_state', 'cell_state'], ['output0'], [0]), ('Squeeze', ('output0', 4), ['output1'], [[1]]), ('Squeeze', ('output0', 4), ['output1'], [[1]]), ('Transpose', ['output1'], [[2, 1, 3]])]
#:set inputs = [['output0', 4], ['output1', 3]]
#:set trueInputs = [['input', [1, 25, 10]], ['hidden_state', [1, 1, 20]], ['cell_state', [1, 1, 20]]]
#:set outShape = [['output', [1, 25, 20]]]
#:set outputs = {'output': 'output1'}
